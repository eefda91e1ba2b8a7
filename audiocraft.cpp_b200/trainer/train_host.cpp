// Host-side training controls; see train_host.h.
#include "train_host.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iomanip>
#include <limits>
#include <map>
#include <set>
#include <sstream>

namespace actf {

void check(act_ctx* ctx, int rc, const char* what) {
    if (rc != ACT_OK) throw std::runtime_error(std::string(what) + ": " + act_last_error(ctx));
}

std::vector<std::string> gguf_files(const std::string& directory) {
    std::vector<std::string> paths;
    for (const auto& entry : std::filesystem::directory_iterator(directory))
        if (entry.is_regular_file() && entry.path().extension() == ".gguf") paths.push_back(entry.path().string());
    std::sort(paths.begin(), paths.end());
    return paths;
}

int parse_device(const std::string& d) {
    if (d == "gpu" || d == "cuda") return 0;
    for (const std::string pre : {"gpu:", "cuda:"})
        if (d.rfind(pre, 0) == 0) return std::stoi(d.substr(pre.size()));
    if (d == "cpu") throw std::runtime_error("this trainer runs the step on a CUDA device; use --device gpu");
    throw std::runtime_error("unknown device: " + d);
}

void save_adapter(act_ctx* ctx, const std::string& path, const std::function<void(GgufWriter&)>& meta) {
    if (std::filesystem::exists(path)) throw std::runtime_error("refusing to overwrite adapter: " + path);
    const auto params = read_params(ctx, false);
    GgufWriter g;
    meta(g);
    for (const auto& p : params) g.add_f32_tensor(p.name, {p.cols, p.rows}, p.value.data());
    g.write(path);
}

std::vector<LoadedLora> load_lora(const GgufReader& base, const GgufReader& adapter, float strength,
                                  const std::string& family) {
    const std::string want = family == "dit" ? "ac-melodyflow-lora" : "ac-musicgen-lora";
    if (adapter.string("general.architecture") != want)
        throw GgufError(family == "dit" ? "not a MelodyFlow adapter" : "not a MusicGen adapter");
    if (adapter.u32("ac.lora.version") != 1) throw GgufError("unsupported adapter");
    const int rank = (int)adapter.u32("ac.lora.rank");
    const float alpha = adapter.f32("ac.lora.alpha");
    const std::string type = adapter.has("ac.lora.type") ? adapter.string("ac.lora.type") : "lora";
    if (type != "lora" && type != "dora-rows") throw GgufError("unsupported adapter type: " + type);
    const bool dora = type == "dora-rows";
    if (rank <= 0 || !std::isfinite(alpha) || alpha <= 0 || !std::isfinite(strength))
        throw GgufError("invalid adapter rank, alpha or strength");
    auto ends_with = [](const std::string& x, const std::string& tail) {
        return x.size() > tail.size() && x.compare(x.size() - tail.size(), tail.size(), tail) == 0;
    };
    std::map<std::string, LoadedLora> out;
    for (const auto& t : adapter.tensors()) {
        if (!ends_with(t.name, ".lora_A")) continue;
        const std::string stem = t.name.substr(0, t.name.size() - 7);
        const GgufTensor& B = adapter.get(stem + ".lora_B");
        const GgufTensor& W = base.get(stem);
        const bool w2d = W.ne[1] > 1 && W.ne[2] == 1 && W.ne[3] == 1;
        if (t.type != GT_F32 || B.type != GT_F32 || !w2d || t.ne[0] != W.ne[0] || t.ne[1] != rank ||
            B.ne[0] != rank || B.ne[1] != W.ne[1] || t.ne[2] != 1 || t.ne[3] != 1 || B.ne[2] != 1 || B.ne[3] != 1)
            throw GgufError("adapter shape mismatch: " + stem);
        LoadedLora p;
        p.stem = stem;
        p.A = &t;
        p.B = &B;
        p.scale = (dora ? 1 : strength) * alpha / rank;
        if (dora) {
            const GgufTensor& m = adapter.get(stem + ".magnitude");
            if (m.type != GT_F32 || m.ne[0] != W.ne[1] || m.ne[1] != 1 || m.ne[2] != 1 || m.ne[3] != 1)
                throw GgufError("DoRA magnitude shape mismatch: " + stem);
            if (W.type != GT_F32 && W.type != GT_F16 && W.type != GT_Q8_0)
                throw GgufError("DoRA rows requires F16/F32/Q8_0 matrix weights");
            p.magnitude = &m;
            p.strength = strength;
        }
        out[stem] = p;
    }
    if (out.empty() || adapter.tensors().size() != (dora ? 3 : 2) * out.size())
        throw GgufError("empty or incomplete adapter");
    for (const auto& e : out)
        for (const GgufTensor* t : {e.second.A, e.second.B, e.second.magnitude}) {
            if (!t) continue;
            const float* v = reinterpret_cast<const float*>(t->data);
            for (int64_t i = 0; i < t->nelements(); ++i)
                if (!std::isfinite(v[i])) throw GgufError("nonfinite adapter tensor");
        }
    if (adapter.has("ac.lora.base_name") && adapter.string("ac.lora.base_name") != base.string("general.name"))
        throw GgufError("adapter base model name does not match");
    static const char* kSuffixes[] = {".self.qkv.weight", ".self.out.weight", ".cross.q.weight", ".cross.kv.weight",
                                      ".cross.out.weight", ".ff.0.weight", ".ff.2.weight"};
    std::vector<LoadedLora> result;
    for (const auto& e : out) {
        bool supported = false;
        for (const char* suffix : kSuffixes)
            supported |= e.first.rfind(family + ".", 0) == 0 && ends_with(e.first, suffix);
        if (!supported)
            throw GgufError(std::string(family == "dit" ? "unsupported MelodyFlow" : "unsupported MusicGen") +
                            " adapter target: " + e.first);
        result.push_back(e.second);
    }
    return result;
}

// ------------------------------------------------------------------ controls and schedule
void TrainControls::validate() const {
    if (accumulation <= 0 || warmup < 0 || !std::isfinite(beta1) || beta1 < 0 || beta1 >= 1 ||
        !std::isfinite(beta2) || beta2 < 0 || beta2 >= 1 || !std::isfinite(eps) || eps <= 0 ||
        !std::isfinite(decay) || decay < 0 || !std::isfinite(clip) || clip <= 0 ||
        (schedule != "constant" && schedule != "inverse"))
        throw std::runtime_error("invalid optimizer controls");
}

float TrainControls::rate(float lr, int step) const {
    float factor = warmup ? std::min(1.f, float(step) / warmup) : 1.f;
    if (schedule == "inverse") factor *= std::pow(1.f + float(step - 1) / 1000000.f, -.5f);
    return lr * factor;
}

std::string TrainControls::signature(float lr) const {
    std::ostringstream o;
    o << std::setprecision(9) << accumulation << ' ' << warmup << ' ' << beta1 << ' ' << beta2 << ' ' << eps << ' '
      << decay << ' ' << clip << ' ' << schedule << ' ' << feedforward << ' ' << random_crop << ' ' << lr;
    return o.str();
}

const char* TrainControls::help() {
    return "  --accumulation-steps N --warmup-steps N --lr-schedule constant|inverse\n"
           "  --beta1 F --beta2 F --adam-eps F --weight-decay F --grad-clip F\n"
           "  --train-ffn (also adapt feed-forward projections)\n"
           "  --random-crop (fresh training crops; validation center crops)\n"
           "  --eval-unconditional (null-text probes) --resume FILE.state\n";
}

act_opt TrainControls::opt(float lr, int step, int count) const {
    act_opt o;
    o.lr = lr;
    o.beta1 = beta1;
    o.beta2 = beta2;
    o.eps = eps;
    o.weight_decay = decay;
    o.clip = clip;
    o.step = step;
    o.count = count;
    return o;
}

// ------------------------------------------------------------------ time sampler
MfTimeSampler::MfTimeSampler(std::string kind_, float mean_, float stddev_)
    : kind(std::move(kind_)), mean(mean_), stddev(stddev_) {
    if ((kind != "uniform" && kind != "logit-normal") || !std::isfinite(mean) || !std::isfinite(stddev) ||
        stddev <= 0)
        throw std::runtime_error("invalid timestep sampling settings");
}

float MfTimeSampler::sample(std::mt19937& rng) const {
    if (kind == "uniform") return std::uniform_real_distribution<float>(0, 1)(rng);
    const float z = std::normal_distribution<float>(mean, stddev)(rng);
    // the logistic of z, written so that neither branch overflows
    const float e = std::exp(-std::fabs(z));
    return std::clamp(z >= 0 ? 1 / (1 + e) : e / (1 + e), 1e-6f, 1 - 1e-6f);
}

// ------------------------------------------------------------------ parameters through the ABI
std::vector<HostParam> read_params(act_ctx* ctx, bool moments) {
    const int64_t n = act_param_count(ctx);
    const int nt = act_param_tensor_count(ctx);
    if (n < 0 || nt < 0) throw std::runtime_error(std::string("parameter table: ") + act_last_error(ctx));
    std::vector<float> value((size_t)n), m(moments ? (size_t)n : 0), v(moments ? (size_t)n : 0);
    check(ctx, act_get_params(ctx, value.data(), moments ? m.data() : nullptr, moments ? v.data() : nullptr, (size_t)n),
          "act_get_params");
    std::vector<HostParam> out((size_t)nt);
    for (int i = 0; i < nt; ++i) {
        char name[256];
        auto& p = out[(size_t)i];
        check(ctx, act_param_tensor(ctx, i, name, sizeof(name), &p.offset, &p.rows, &p.cols), "act_param_tensor");
        p.name = name;
        const size_t cnt = (size_t)(p.rows * p.cols);
        p.value.assign(value.begin() + p.offset, value.begin() + p.offset + cnt);
        p.m = moments ? std::vector<float>(m.begin() + p.offset, m.begin() + p.offset + cnt) : std::vector<float>(cnt, 0.f);
        p.v = moments ? std::vector<float>(v.begin() + p.offset, v.begin() + p.offset + cnt) : std::vector<float>(cnt, 0.f);
    }
    return out;
}

void write_params(act_ctx* ctx, const std::vector<HostParam>& params) {
    const int64_t n = act_param_count(ctx);
    std::vector<float> value((size_t)n), m((size_t)n), v((size_t)n);
    for (const auto& p : params) {
        std::copy(p.value.begin(), p.value.end(), value.begin() + p.offset);
        std::copy(p.m.begin(), p.m.end(), m.begin() + p.offset);
        std::copy(p.v.begin(), p.v.end(), v.begin() + p.offset);
    }
    check(ctx, act_set_params(ctx, value.data(), (size_t)n), "act_set_params");
    check(ctx, act_set_moments(ctx, m.data(), v.data(), (size_t)n), "act_set_moments");
}

// ------------------------------------------------------------------ exact-resume state
void train_state(const std::string& path, bool load, const std::string& signature, std::vector<HostParam>& params,
                 int& step, size_t& seen, std::mt19937& rng, std::vector<size_t>& order) {
    std::fstream f;
    if (!load && std::filesystem::exists(path)) throw std::runtime_error("trainer state already exists");
    const std::string temporary = path + ".tmp";
    f.open(load ? path : temporary, load ? std::ios::in : std::ios::out);
    if (!f) throw std::runtime_error("cannot open trainer state: " + path);
    f << std::setprecision(std::numeric_limits<float>::max_digits10);
    auto scalar = [&](auto& v) {
        if (load) f >> v;
        else f << v << '\n';
    };
    std::string tag = "ac-trainer-state-v1", sig = signature;
    if (load) {
        f >> std::quoted(tag) >> std::quoted(sig);
        if (tag != "ac-trainer-state-v1" || sig != signature)
            throw std::runtime_error("trainer state configuration/data mismatch");
    } else {
        f << std::quoted(tag) << '\n' << std::quoted(sig) << '\n';
    }
    scalar(step);
    scalar(seen);
    scalar(rng);
    size_t n = order.size();
    scalar(n);
    if (n != order.size()) throw std::runtime_error("trainer state order mismatch");
    for (auto& v : order) scalar(v);
    auto sorted = order;
    std::sort(sorted.begin(), sorted.end());
    for (size_t i = 0; i < sorted.size(); ++i)
        if (sorted[i] != i) throw std::runtime_error("invalid trainer sample order");
    n = params.size();
    scalar(n);
    if (n != params.size()) throw std::runtime_error("trainer state parameter count mismatch");
    for (auto& p : params) {
        std::string name = p.name;
        if (load) {
            f >> std::quoted(name);
            if (name != p.name) throw std::runtime_error("trainer state parameter mismatch");
        } else {
            f << std::quoted(name) << '\n';
        }
        n = p.value.size();
        scalar(n);
        if (n != p.value.size()) throw std::runtime_error("trainer state shape mismatch");
        for (auto* vec : {&p.value, &p.m, &p.v})
            for (auto& x : *vec) {
                scalar(x);
                if (!std::isfinite(x)) throw std::runtime_error("nonfinite trainer state");
            }
    }
    if (!f) throw std::runtime_error("truncated/unwritable trainer state");
    if (load) {
        f >> std::ws;
        if (!f.eof()) throw std::runtime_error("trailing trainer state data");
    } else {
        f.flush();
        if (!f) throw std::runtime_error("trainer state flush failed");
        f.close();
        std::filesystem::rename(temporary, path);
    }
}

std::string train_file_identity(const std::string& file) {
    std::ifstream f(file, std::ios::binary);
    if (!f) throw std::runtime_error("cannot fingerprint " + file);
    uint64_t h = 14695981039346656037ull;  // FNV-1a 64 offset basis
    std::vector<char> buf(1 << 16);
    while (f) {
        f.read(buf.data(), (std::streamsize)buf.size());
        for (std::streamsize i = 0; i < f.gcount(); ++i) {
            h ^= (unsigned char)buf[(size_t)i];
            h *= 1099511628211ull;  // FNV prime
        }
    }
    if (!f.eof()) throw std::runtime_error("fingerprint read failed");
    return std::to_string(h);
}

std::string key_part(float v) {
    std::ostringstream o;
    o << std::setprecision(std::numeric_limits<float>::max_digits10) << v;
    return o.str();
}
std::string key_part(int v) { return std::to_string(v); }
std::string key_part(uint32_t v) { return std::to_string(v); }
std::string key_part(const std::string& v) { return v; }

std::string train_key_join(const std::vector<std::string>& parts) {
    std::string out;
    for (const auto& p : parts) out += p + '|';
    return out;
}

// ------------------------------------------------------------------ caption pool (JSON)
namespace {

struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    bool is_uint = false;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json* get(const std::string& k) const {
        for (const auto& kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JsonParser {
    const std::string& s;
    size_t i = 0;
    [[noreturn]] void fail() const { throw std::runtime_error("invalid JSON"); }
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (s.compare(i, n, w) != 0) return false;
        i += n;
        return true;
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) out += (char)cp;
        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 63)); }
        else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
        } else {
            out += (char)(0xF0 | (cp >> 18)); out += (char)(0x80 | ((cp >> 12) & 63));
            out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63));
        }
    }
    uint32_t hex4() {
        if (i + 4 > s.size()) fail();
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s[i++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail();
        }
        return v;
    }
    std::string string() {
        if (s[i] != '"') fail();
        ++i;
        std::string out;
        while (true) {
            if (i >= s.size()) fail();
            const char c = s[i++];
            if (c == '"') break;
            if ((unsigned char)c < 0x20) fail();
            if (c != '\\') { out += c; continue; }
            if (i >= s.size()) fail();
            const char e = s[i++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00) {
                        if (!lit("\\u")) fail();
                        const uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo >= 0xE000) fail();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail();
            }
        }
        return out;
    }
    Json value(int depth) {
        if (depth > 64) fail();
        ws();
        if (i >= s.size()) fail();
        Json j;
        const char c = s[i];
        if (c == '{') {
            j.kind = Json::Obj;
            ++i;
            ws();
            if (i < s.size() && s[i] == '}') { ++i; return j; }
            while (true) {
                ws();
                std::string k = string();
                ws();
                if (i >= s.size() || s[i++] != ':') fail();
                j.obj.emplace_back(std::move(k), value(depth + 1));
                ws();
                if (i >= s.size()) fail();
                if (s[i] == ',') { ++i; continue; }
                if (s[i++] != '}') fail();
                return j;
            }
        }
        if (c == '[') {
            j.kind = Json::Arr;
            ++i;
            ws();
            if (i < s.size() && s[i] == ']') { ++i; return j; }
            while (true) {
                j.arr.push_back(value(depth + 1));
                ws();
                if (i >= s.size()) fail();
                if (s[i] == ',') { ++i; continue; }
                if (s[i++] != ']') fail();
                return j;
            }
        }
        if (c == '"') { j.kind = Json::Str; j.str = string(); return j; }
        if (lit("true")) { j.kind = Json::Bool; j.b = true; return j; }
        if (lit("false")) { j.kind = Json::Bool; return j; }
        if (lit("null")) return j;
        const size_t start = i;
        if (s[i] == '-') ++i;
        bool frac = false;
        while (i < s.size() && (std::isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                                s[i] == '+' || s[i] == '-')) {
            if (!std::isdigit((unsigned char)s[i])) frac = true;
            ++i;
        }
        if (i == start) fail();
        j.kind = Json::Num;
        j.num = std::stod(s.substr(start, i - start));
        j.is_uint = !frac && s[start] != '-';
        return j;
    }
};

void json_escape(std::string& out, const std::string& s) {
    // ASCII output: control characters and every non-ASCII code point as \uXXXX (UTF-16)
    auto u16 = [&](uint32_t v) {
        char b[16];
        std::snprintf(b, sizeof(b), "\\u%04X", v & 0xFFFFu);
        out += b;
    };
    out += '"';
    for (size_t i = 0; i < s.size();) {
        const unsigned char c = (unsigned char)s[i];
        if (c < 0x80) {
            ++i;
            switch (c) {
                case '"': out += "\\\""; break;
                case '\\': out += "\\\\"; break;
                case '\b': out += "\\b"; break;
                case '\f': out += "\\f"; break;
                case '\n': out += "\\n"; break;
                case '\r': out += "\\r"; break;
                case '\t': out += "\\t"; break;
                default:
                    if (c < 0x20) u16(c);
                    else out += (char)c;
            }
            continue;
        }
        int len = c >= 0xF0 ? 4 : c >= 0xE0 ? 3 : c >= 0xC0 ? 2 : 0;
        if (!len || i + len > s.size()) throw std::runtime_error("invalid UTF-8 caption");
        uint32_t cp = c & (0x3F >> (len - 1));
        for (int k = 1; k < len; ++k) {
            const unsigned char d = (unsigned char)s[i + k];
            if ((d & 0xC0) != 0x80) throw std::runtime_error("invalid UTF-8 caption");
            cp = (cp << 6) | (d & 63);
        }
        i += len;
        if (cp >= 0x10000) {
            cp -= 0x10000;
            u16(0xD800 + (cp >> 10));
            u16(0xDC00 + (cp & 0x3FF));
        } else {
            u16(cp);
        }
    }
    out += '"';
}

}  // namespace

std::string prompt_pool_path(const std::string& adapter) {
    auto p = std::filesystem::path(adapter);
    p.replace_extension(".prompts.json");
    return p.string();
}

std::vector<std::string> read_prompt_pool(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot read prompt pool: " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    Json root;
    try {
        JsonParser p{text};
        root = p.value(0);
        p.ws();
        if (p.i != text.size()) p.fail();
    } catch (const std::exception&) {
        throw std::runtime_error("cannot read prompt pool: " + path);
    }
    const Json* version = root.kind == Json::Obj ? root.get("version") : nullptr;
    const Json* dice = root.kind == Json::Obj ? root.get("dice") : nullptr;
    const Json* prompts = dice && dice->kind == Json::Obj ? dice->get("instrumental") : nullptr;
    if (!version || version->kind != Json::Num || !version->is_uint || version->num != 1 || !prompts ||
        prompts->kind != Json::Arr)
        throw std::runtime_error("unsupported prompt pool: " + path);
    std::vector<std::string> result;
    for (const auto& item : prompts->arr) {
        if (item.kind != Json::Str || item.str.empty()) throw std::runtime_error("invalid prompt pool caption");
        result.push_back(item.str);
    }
    if (result.empty()) throw std::runtime_error("prompt pool is empty");
    return result;
}

void write_prompt_pool(const std::string& path, const std::string& adapter, const std::vector<std::string>& captions,
                       size_t files) {
    if (std::filesystem::exists(path)) throw std::runtime_error("refusing to overwrite prompt pool: " + path);
    std::set<std::string> seen;
    std::vector<std::string> unique;
    for (const auto& c : captions)
        if (!c.empty() && seen.insert(c).second) unique.push_back(c);
    if (seen.empty()) throw std::runtime_error("training captions contain no nonempty prompts");
    // 4-space pretty printing, keys in the reference's order
    std::string out = "{\n    \"version\": 1,\n    \"source\": {\n        \"lora\": ";
    json_escape(out, std::filesystem::path(adapter).filename().string());
    out += ",\n        \"files\": " + std::to_string(files) + ",\n        \"unique_prompts\": " +
           std::to_string(seen.size()) + "\n    },\n    \"dice\": {\n        \"instrumental\": [";
    for (size_t i = 0; i < unique.size(); ++i) {
        out += i ? ",\n            " : "\n            ";
        json_escape(out, unique[i]);
    }
    out += "\n        ]\n    }\n}";
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot write prompt pool: " + path);
    f << out;
    f.close();
    if (!f) throw std::runtime_error("cannot write prompt pool: " + path);
}

}  // namespace actf
