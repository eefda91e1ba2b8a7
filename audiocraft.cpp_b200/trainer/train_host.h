// Host-side training controls shared by mf-train and mg-train: optimizer flags and the learning
// rate schedule, the time sampler, the exact-resume state file, file fingerprints and the caption
// pool.  These follow the reference's host code (src/ac/train_controls.h, src/mf/train.h:14-29,
// src/ac/prompt_pool.h); the device work goes through the act_* C ABI.
#pragma once
#include <cstdint>
#include <functional>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "actrain.h"
#include "gguf_file.h"

namespace actf {

// Optimizer and loop flags (TrainControls, src/ac/train_controls.h:12-72).
struct TrainControls {
    int accumulation = 1, warmup = 0;
    float beta1 = .9f, beta2 = .999f, eps = 1e-8f, decay = 0, clip = 1;
    std::string schedule = "constant", resume;
    bool feedforward = false, random_crop = false, eval_null = false;

    // consumes one flag (and its value through next()); false when the flag is not one of these
    template <class Next>
    bool parse(const std::string& a, Next next);
    void validate() const;
    // warm-up ramp min(1, step/warmup), then optionally (1 + (step-1)/1e6)^-1/2 (src/ac/train_controls.h:53-58)
    float rate(float lr, int step) const;
    // the flags that must agree for a resume (src/ac/train_controls.h:59-65)
    std::string signature(float lr) const;
    static const char* help();
    // AdamW settings of one update (TrainAccumulation::update, src/ac/train_controls.h:89-118)
    act_opt opt(float lr, int step, int count) const;
};

// Training flow time: uniform, or logit-normal clamped to [1e-6, 1-1e-6] (MfTimeSampler,
// src/mf/train.h:14-29).  Validation stays uniform / stratified.
struct MfTimeSampler {
    std::string kind;
    float mean, stddev;
    explicit MfTimeSampler(std::string kind = "uniform", float mean = 0, float stddev = 1);
    float sample(std::mt19937& rng) const;
};

// One adapter tensor on the host: what the adapter file and the state file hold.
struct HostParam {
    std::string name;
    int64_t offset = 0, rows = 0, cols = 0;  // in the flat parameter vector; [rows][cols]
    std::vector<float> value, m, v;
};

// The context's parameter table and values (act_param_tensor / act_get_params).
std::vector<HostParam> read_params(act_ctx* ctx, bool moments);
// Upload values and moments (resume).
void write_params(act_ctx* ctx, const std::vector<HostParam>& params);

// Exact-resume state, written only at optimizer-update boundaries; load checks the signature,
// the sample order and every parameter name and size (train_state, src/ac/train_controls.h:122-196).
void train_state(const std::string& path, bool load, const std::string& signature, std::vector<HostParam>& params,
                 int& step, size_t& seen, std::mt19937& rng, std::vector<size_t>& order);

// 64-bit FNV-1a of a file's bytes, as decimal (train_file_identity, src/ac/train_controls.h:206-221)
std::string train_file_identity(const std::string& file);

// values joined with '|' at float round-trip precision (train_key, src/ac/train_controls.h:198-204)
std::string train_key_join(const std::vector<std::string>& parts);
std::string key_part(float v);
std::string key_part(int v);
std::string key_part(uint32_t v);
std::string key_part(const std::string& v);
template <class... T>
std::string train_key(const T&... values) {
    return train_key_join({key_part(values)...});
}

// Caption pool beside the adapter (src/ac/prompt_pool.h:12-84).
std::string prompt_pool_path(const std::string& adapter);
std::vector<std::string> read_prompt_pool(const std::string& path);
void write_prompt_pool(const std::string& path, const std::string& adapter, const std::vector<std::string>& captions,
                       size_t files);

// The ABI's status as an exception (the CLIs report it and return 1).
void check(act_ctx* ctx, int rc, const char* what);

// The *.gguf files of a directory, sorted by path (the reference's cache order).
std::vector<std::string> gguf_files(const std::string& directory);
// "gpu" / "cuda" (device 0) or "gpu:N" / "cuda:N"; "cpu" is refused: the step runs on a GPU.
int parse_device(const std::string& device);
// An adapter file: `meta` sets the keys, then every parameter tensor follows as F32 in the
// reference's order and shape (MfTrainGraph::save / MgTrainGraph::save); an existing file is kept.
void save_adapter(act_ctx* ctx, const std::string& path, const std::function<void(GgufWriter&)>& meta);

// One adapted projection of a validated adapter file (LoraProjection, src/ac/lora.h:38-47).
struct LoadedLora {
    std::string stem;  // the base weight's name, e.g. dit.3.self.qkv.weight
    const GgufTensor* A = nullptr;          // [rank][in]
    const GgufTensor* B = nullptr;          // [out][rank]
    const GgufTensor* magnitude = nullptr;  // [out] (DoRA rows) or null
    float scale = 1.0f;                     // (DoRA ? 1 : strength) * alpha / rank
    float strength = 1.0f;
};

// load_mf_lora / load_mg_lora (src/ac/lora.h:113-210): checks an adapter file against its base
// model -- architecture and version, rank / alpha / type, every tensor's shape against the base
// weight, completeness, finite values, the base model's name, the supported targets of the family
// ("dit" for MelodyFlow, "lm" for MusicGen) -- and returns its projections in name order.
// Unlike the reference, DoRA rows may sit on a Q8_0 base (this library trains them).
std::vector<LoadedLora> load_lora(const GgufReader& base, const GgufReader& adapter, float strength,
                                  const std::string& family);

template <class Next>
bool TrainControls::parse(const std::string& a, Next next) {
    if (a == "--accumulation-steps") accumulation = std::stoi(next());
    else if (a == "--warmup-steps") warmup = std::stoi(next());
    else if (a == "--lr-schedule") schedule = next();
    else if (a == "--beta1") beta1 = std::stof(next());
    else if (a == "--beta2") beta2 = std::stof(next());
    else if (a == "--adam-eps") eps = std::stof(next());
    else if (a == "--weight-decay") decay = std::stof(next());
    else if (a == "--grad-clip") clip = std::stof(next());
    else if (a == "--train-ffn") feedforward = true;
    else if (a == "--random-crop") random_crop = true;
    else if (a == "--eval-unconditional") eval_null = true;
    else if (a == "--resume") resume = next();
    else return false;
    return true;
}

}  // namespace actf
