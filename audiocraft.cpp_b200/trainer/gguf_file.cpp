// GGUF reader (mapped, bounds-checked) and writer; the format is described in gguf_file.h.
#include "gguf_file.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>

namespace actf {

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" little-endian
constexpr uint32_t kDefaultAlignment = 32;

struct Cursor {
    const uint8_t* p;
    size_t n, at = 0;
    const std::string& path;
    void need(size_t k) const {
        if (k > n - at) throw GgufError("truncated file: " + path);
    }
    template <class T>
    T pod() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t len = pod<uint64_t>();
        need(len);
        std::string s(reinterpret_cast<const char*>(p + at), len);
        at += len;
        return s;
    }
};

GgufValue read_value(Cursor& c, uint32_t type, int depth) {
    GgufValue v;
    v.type = type;
    switch (type) {
        case GV_U8: v.u = c.pod<uint8_t>(); break;
        case GV_I8: v.i = c.pod<int8_t>(); break;
        case GV_U16: v.u = c.pod<uint16_t>(); break;
        case GV_I16: v.i = c.pod<int16_t>(); break;
        case GV_U32: v.u = c.pod<uint32_t>(); break;
        case GV_I32: v.i = c.pod<int32_t>(); break;
        case GV_F32: v.f = c.pod<float>(); break;
        case GV_BOOL: {
            const uint8_t b = c.pod<uint8_t>();
            if (b > 1) throw GgufError("invalid bool value: " + c.path);
            v.u = b;
            break;
        }
        case GV_STRING: v.s = c.str(); break;
        case GV_U64: v.u = c.pod<uint64_t>(); break;
        case GV_I64: v.i = c.pod<int64_t>(); break;
        case GV_F64: v.f = c.pod<double>(); break;
        case GV_ARRAY: {
            if (depth > 0) throw GgufError("nested arrays are not supported: " + c.path);
            v.elem = c.pod<uint32_t>();
            const uint64_t n = c.pod<uint64_t>();
            if (n > c.n) throw GgufError("invalid array length: " + c.path);
            v.arr.reserve(n);
            for (uint64_t k = 0; k < n; ++k) v.arr.push_back(read_value(c, v.elem, depth + 1));
            break;
        }
        default: throw GgufError("unknown value type " + std::to_string(type) + ": " + c.path);
    }
    return v;
}

const char* type_name(uint32_t t) {
    switch (t) {
        case GV_U32: return "u32";
        case GV_F32: return "f32";
        case GV_BOOL: return "bool";
        case GV_STRING: return "string";
        default: return "other";
    }
}

template <class T>
void put(std::string& out, const T& v) {
    out.append(reinterpret_cast<const char*>(&v), sizeof(T));
}

void put_str(std::string& out, const std::string& s) {
    put<uint64_t>(out, s.size());
    out += s;
}

int ggml_n_dims(const std::vector<int64_t>& ne) {
    int n = 1;
    for (int d = (int)ne.size() - 1; d >= 1; --d)
        if (ne[d] > 1) { n = d + 1; break; }
    return n;
}

size_t pad_to(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace

int64_t GgufTensor::nelements() const {
    int64_t n = 1;
    for (int64_t e : ne) n *= e;
    return n;
}

size_t ggml_type_bytes(uint32_t type, int64_t n) {
    switch (type) {
        case GT_F32:
        case GT_I32: return (size_t)n * 4;
        case GT_F16:
        case GT_BF16: return (size_t)n * 2;
        case GT_Q8_0:
            if (n % 32) throw GgufError("Q8_0 tensor size is not a multiple of 32");
            return (size_t)(n / 32) * 34;
        default: throw GgufError("unsupported tensor type " + std::to_string(type));
    }
}

GgufReader::GgufReader(const std::string& path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw GgufError("cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) {
        ::close(fd_);
        throw GgufError("cannot stat " + path);
    }
    size_ = (size_t)st.st_size;
    if (size_ < 24) {
        ::close(fd_);
        throw GgufError("not a GGUF file: " + path);
    }
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) {
        ::close(fd_);
        throw GgufError("cannot map " + path);
    }
    map_ = static_cast<const uint8_t*>(m);
    try {
        Cursor c{map_, size_, 0, path_};
        if (c.pod<uint32_t>() != kMagic) throw GgufError("not a GGUF file: " + path);
        const uint32_t version = c.pod<uint32_t>();
        if (version != 2 && version != 3) throw GgufError("unsupported GGUF version " + std::to_string(version));
        const int64_t nt = c.pod<int64_t>(), nkv = c.pod<int64_t>();
        if (nt < 0 || nkv < 0 || (uint64_t)nt > size_ || (uint64_t)nkv > size_) throw GgufError("invalid counts: " + path);
        for (int64_t k = 0; k < nkv; ++k) {
            std::string key = c.str();
            const uint32_t type = c.pod<uint32_t>();
            GgufValue v = read_value(c, type, 0);
            if (!kv_.emplace(key, std::move(v)).second) throw GgufError("duplicate key " + key + ": " + path);
        }
        uint32_t alignment = kDefaultAlignment;
        if (has("general.alignment")) {
            alignment = u32("general.alignment");
            if (alignment == 0 || (alignment & (alignment - 1))) throw GgufError("invalid alignment: " + path);
        }
        for (int64_t k = 0; k < nt; ++k) {
            GgufTensor t;
            t.name = c.str();
            const uint32_t nd = c.pod<uint32_t>();
            if (nd == 0 || nd > 4) throw GgufError("invalid tensor rank: " + t.name);
            for (uint32_t d = 0; d < nd; ++d) {
                const int64_t e = c.pod<int64_t>();
                if (e < 0) throw GgufError("invalid tensor shape: " + t.name);
                t.ne.push_back(e);
            }
            while (t.ne.size() < 4) t.ne.push_back(1);
            t.type = c.pod<uint32_t>();
            t.offset = c.pod<uint64_t>();
            if (t.offset % alignment) throw GgufError("misaligned tensor data: " + t.name);
            if (!index_.emplace(t.name, tensors_.size()).second) throw GgufError("duplicate tensor " + t.name);
            tensors_.push_back(std::move(t));
        }
        const size_t data0 = pad_to(c.at, alignment);
        for (auto& t : tensors_) {
            t.bytes = ggml_type_bytes(t.type, t.nelements());
            if (data0 > size_ || t.offset > size_ - data0 || t.bytes > size_ - data0 - t.offset)
                throw GgufError("tensor data out of range: " + t.name);
            t.data = map_ + data0 + t.offset;
        }
    } catch (...) {
        munmap(const_cast<uint8_t*>(map_), size_);
        ::close(fd_);
        throw;
    }
}

GgufReader::~GgufReader() {
    if (map_) munmap(const_cast<uint8_t*>(map_), size_);
    if (fd_ >= 0) ::close(fd_);
}

const GgufValue& GgufReader::value(const std::string& key) const {
    auto it = kv_.find(key);
    if (it == kv_.end()) throw GgufError("missing key " + key + " in " + path_);
    return it->second;
}

std::string GgufReader::string(const std::string& key) const {
    const auto& v = value(key);
    if (v.type != GV_STRING) throw GgufError(key + " is " + type_name(v.type) + ", expected string");
    return v.s;
}

uint32_t GgufReader::u32(const std::string& key) const {
    const auto& v = value(key);
    if (v.type != GV_U32) throw GgufError(key + " is " + type_name(v.type) + ", expected u32");
    return (uint32_t)v.u;
}

float GgufReader::f32(const std::string& key) const {
    const auto& v = value(key);
    if (v.type != GV_F32) throw GgufError(key + " is " + type_name(v.type) + ", expected f32");
    return (float)v.f;
}

bool GgufReader::boolean(const std::string& key) const {
    const auto& v = value(key);
    if (v.type != GV_BOOL) throw GgufError(key + " is " + type_name(v.type) + ", expected bool");
    return v.u != 0;
}

const GgufTensor* GgufReader::find(const std::string& name) const {
    auto it = index_.find(name);
    return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GgufTensor& GgufReader::get(const std::string& name) const {
    const GgufTensor* t = find(name);
    if (!t) throw GgufError("missing tensor " + name + " in " + path_);
    return *t;
}

std::vector<float> GgufReader::read_f32(const std::string& name) const {
    const GgufTensor& t = get(name);
    if (t.type != GT_F32) throw GgufError("training cache must be F32");
    std::vector<float> v((size_t)t.nelements());
    std::memcpy(v.data(), t.data, v.size() * 4);
    for (float x : v)
        if (!std::isfinite(x)) throw GgufError("nonfinite training tensor");
    return v;
}

void GgufWriter::add_kv(const std::string& key, uint32_t type, std::string bytes) {
    for (auto& k : kv_)
        if (k.key == key) {  // gguf_set_val_*: a key set twice keeps its place, takes the new value
            k.type = type;
            k.bytes = std::move(bytes);
            return;
        }
    kv_.push_back({key, type, std::move(bytes)});
}

void GgufWriter::add_string(const std::string& key, const std::string& v) {
    std::string b;
    put_str(b, v);
    add_kv(key, GV_STRING, std::move(b));
}

void GgufWriter::add_u32(const std::string& key, uint32_t v) {
    std::string b;
    put(b, v);
    add_kv(key, GV_U32, std::move(b));
}

void GgufWriter::add_f32(const std::string& key, float v) {
    std::string b;
    put(b, v);
    add_kv(key, GV_F32, std::move(b));
}

void GgufWriter::add_bool(const std::string& key, bool v) {
    std::string b;
    put<uint8_t>(b, v ? 1 : 0);
    add_kv(key, GV_BOOL, std::move(b));
}

void GgufWriter::add_f32_tensor(const std::string& name, const std::vector<int64_t>& ne, const float* data) {
    int64_t n = 1;
    for (int64_t e : ne) n *= e;
    tensors_.push_back({name, ne, GT_F32, std::string(reinterpret_cast<const char*>(data), (size_t)n * 4)});
}

void GgufWriter::add_i32_tensor(const std::string& name, const std::vector<int64_t>& ne, const int32_t* data) {
    int64_t n = 1;
    for (int64_t e : ne) n *= e;
    tensors_.push_back({name, ne, GT_I32, std::string(reinterpret_cast<const char*>(data), (size_t)n * 4)});
}

void GgufWriter::write(const std::string& path) const {
    if (std::filesystem::exists(path)) throw GgufError("refusing to overwrite " + path);
    std::string out;
    put<uint32_t>(out, kMagic);
    put<uint32_t>(out, 3);
    put<int64_t>(out, (int64_t)tensors_.size());
    put<int64_t>(out, (int64_t)kv_.size());
    for (const auto& k : kv_) {
        put_str(out, k.key);
        put<uint32_t>(out, k.type);
        out += k.bytes;
    }
    uint64_t offset = 0;
    for (const auto& t : tensors_) {
        put_str(out, t.name);
        const int nd = ggml_n_dims(t.ne);
        put<uint32_t>(out, (uint32_t)nd);
        for (int d = 0; d < nd; ++d) put<int64_t>(out, d < (int)t.ne.size() ? t.ne[d] : 1);
        put<uint32_t>(out, t.type);
        put<uint64_t>(out, offset);
        offset += pad_to(t.bytes.size(), kDefaultAlignment);
    }
    out.resize(pad_to(out.size(), kDefaultAlignment), '\0');
    for (const auto& t : tensors_) {
        out += t.bytes;
        out.resize(pad_to(out.size(), kDefaultAlignment), '\0');
    }
    std::ofstream f(path, std::ios::binary);
    if (!f) throw GgufError("cannot write " + path);
    f.write(out.data(), (std::streamsize)out.size());
    f.close();
    if (!f) {
        std::error_code ec;
        std::filesystem::remove(path, ec);
        throw GgufError("failed to write " + path);
    }
}

}  // namespace actf
