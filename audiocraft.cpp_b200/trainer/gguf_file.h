// GGUF v2/v3 files for the trainer front ends: a read-only mapped reader (model weights, training
// caches) and a writer for the adapter files.
//
// The container layout is the published GGUF format that the reference reads and writes through
// ggml's gguf API (load_gguf, src/gguf_model.h:241-346; MfTrainGraph::save, src/mf/train.h:229-255):
//   "GGUF" | u32 version | i64 n_tensors | i64 n_kv | n_kv x (string key, u32 type, value)
//   | n_tensors x (string name, u32 n_dims, i64 ne[n_dims], u32 ggml_type, u64 offset)
//   | zero padding to the alignment | tensor data, each padded to the alignment.
// Strings are a u64 length followed by the bytes.  The alignment is `general.alignment` (u32) when
// present, else 32.  The writer emits keys and tensors in insertion order and records a tensor of
// shape ne with ggml's n_dims rule (1 + the last axis whose extent exceeds 1), as ggml does.
#pragma once
#include <cstdint>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace actf {

// errors carry the reference's "[gguf] " prefix (gguf_error, src/gguf_model.h:29-31)
struct GgufError : std::runtime_error {
    explicit GgufError(const std::string& what) : std::runtime_error("[gguf] " + what) {}
};

enum GgufValueType : uint32_t {
    GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
    GV_STRING = 8, GV_ARRAY = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};

// ggml tensor types the trainers read or write
enum GgmlType : uint32_t { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_I32 = 26, GT_BF16 = 30 };

struct GgufValue {
    uint32_t type = GV_U8;
    uint64_t u = 0;       // unsigned integers and bool
    int64_t i = 0;        // signed integers
    double f = 0;         // f32 / f64
    std::string s;        // string
    uint32_t elem = 0;    // array element type
    std::vector<GgufValue> arr;
};

struct GgufTensor {
    std::string name;
    std::vector<int64_t> ne;  // ggml order: ne[0] is the fastest axis
    uint32_t type = GT_F32;
    uint64_t offset = 0;      // relative to the data section
    const uint8_t* data = nullptr;
    size_t bytes = 0;
    int64_t nelements() const;
};

// bytes of n elements of a ggml type (whole blocks for quantised types); throws for other types
size_t ggml_type_bytes(uint32_t type, int64_t n);

class GgufReader {
public:
    explicit GgufReader(const std::string& path);
    ~GgufReader();
    GgufReader(const GgufReader&) = delete;
    GgufReader& operator=(const GgufReader&) = delete;

    const std::string& path() const { return path_; }
    bool has(const std::string& key) const { return kv_.count(key) != 0; }
    const GgufValue& value(const std::string& key) const;
    // typed accessors: a missing key or a different stored type is an error
    std::string string(const std::string& key) const;
    uint32_t u32(const std::string& key) const;
    float f32(const std::string& key) const;
    bool boolean(const std::string& key) const;

    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    const GgufTensor* find(const std::string& name) const;
    const GgufTensor& get(const std::string& name) const;
    // an F32 tensor as floats, every value finite (train_read_tensor, src/ac/train_utils.h:5-14)
    std::vector<float> read_f32(const std::string& name) const;

private:
    std::string path_;
    int fd_ = -1;
    const uint8_t* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> index_;
};

class GgufWriter {
public:
    void add_string(const std::string& key, const std::string& v);
    void add_u32(const std::string& key, uint32_t v);
    void add_f32(const std::string& key, float v);
    void add_bool(const std::string& key, bool v);
    void add_i32_tensor(const std::string& name, const std::vector<int64_t>& ne, const int32_t* data);
    void add_f32_tensor(const std::string& name, const std::vector<int64_t>& ne, const float* data);
    // writes the whole file; refuses to replace an existing one
    void write(const std::string& path) const;

private:
    struct Kv {
        std::string key;
        uint32_t type;
        std::string bytes;  // encoded value
    };
    struct T {
        std::string name;
        std::vector<int64_t> ne;
        uint32_t type;
        std::string bytes;
    };
    void add_kv(const std::string& key, uint32_t type, std::string bytes);
    std::vector<Kv> kv_;
    std::vector<T> tensors_;
};

}  // namespace actf
