// mf-train on the B200 step: MelodyFlow DiT adapter training from cached latents.
//
// Same flags, sampling, accumulation, checkpoints, adapter file, caption pool and exact-resume
// state as the reference front end (tools/mf-train.cpp:1-359); the forward/backward and AdamW
// run on the GPU through the act_* C ABI instead of a ggml graph.  Every random draw happens on
// the host in the reference's order (shuffle, caption dropout, crop, posterior and noise
// interleaved per element, time), so runs are reproducible and resumable exactly; the draws of
// one optimizer step are batched into as few device microbatches as the context holds.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <filesystem>
#include <set>
#include <string>
#include <vector>

#include "actrain.h"
#include "gguf_file.h"
#include "train_host.h"

namespace {

using actf::GgufReader;

struct DitShape {
    act_model_desc desc{};
    std::string name;  // general.name, when present
};

// DitConfig::from (src/mf/dit.h:44-71)
DitShape dit_config(const GgufReader& m) {
    if (m.string("ac.architecture") != "audiocraft") throw actf::GgufError("not an audiocraft GGUF");
    if (m.u32("ac.format_version") != 1) throw actf::GgufError("unsupported audiocraft GGUF version");
    if (m.string("ac.dit.family") != "melodyflow") throw actf::GgufError("not a MelodyFlow DiT GGUF");
    DitShape s;
    auto& d = s.desc;
    d.family = ACT_FAMILY_MELODYFLOW;
    d.dim = (int)m.u32("ac.dit.dim");
    d.layers = (int)m.u32("ac.dit.layers");
    d.heads = (int)m.u32("ac.dit.heads");
    d.head_dim = (int)m.u32("ac.dit.head_dim");
    d.ff_dim = (int)m.u32("ac.dit.ff_dim");
    d.latent_dim = (int)m.u32("ac.dit.latent_dim");
    d.cond_dim = (int)m.u32("ac.dit.cond_dim");
    d.time_dim = (int)m.u32("ac.dit.time_dim");
    d.n_skip = (int)m.u32("ac.dit.n_skip");
    (void)m.f32("ac.dit.rope_base");  // the stored rope_freq_factors carry the frequencies
    d.norm_eps = m.f32("ac.dit.norm_eps");
    (void)m.f32("ac.dit.cfg_coef");
    (void)m.f32("ac.dit.max_duration");
    d.add_zero_attn = m.boolean("ac.dit.add_zero_attn") ? 1 : 0;
    if (d.dim != d.heads * d.head_dim) throw actf::GgufError("DiT dim does not equal heads * head_dim");
    if (d.n_skip != (d.layers - 1) / 2) throw actf::GgufError("DiT skip count does not match (layers - 1) / 2");
    if (m.has("general.name")) s.name = m.string("general.name");
    return s;
}

struct Sample {
    std::string name, source_id, caption;
    int tokens = 0, frames = 0;
    bool empty = false;
    std::vector<float> mean, stddev, hidden, pivot;
    float edit_start = 0;
};

// read_samples (tools/mf-train.cpp:17-95)
std::vector<Sample> read_samples(const std::string& directory, const GgufReader& model, const act_model_desc& c,
                                 int frames, int& max_tokens, const std::string& objective, float t_min) {
    const auto normalization_mean = model.read_f32("dit.latent_mean");
    auto normalization_std = model.read_f32("dit.latent_std");
    for (auto& v : normalization_std) v += 1e-5f;
    std::vector<Sample> out;
    for (const auto& file : actf::gguf_files(directory)) {
        const std::filesystem::path path(file);
        GgufReader cache(file);
        const bool bridge = objective == "edit-bridge";
        if (cache.string("general.architecture") != (bridge ? "ac-melodyflow-edit-cache" : "ac-melodyflow-train-cache") ||
            cache.u32("ac.cache.version") != 1)
            throw std::runtime_error("unsupported cache: " + path.string());
        if (cache.read_f32("normalization_mean") != normalization_mean ||
            cache.read_f32("normalization_std") != normalization_std)
            throw std::runtime_error("cache normalization does not match the DiT: " + path.string());
        const auto& mean = cache.get("mean");
        const auto& stddev = cache.get("stddev");
        const auto& hidden = cache.get("hidden");
        if (mean.ne[0] < frames || mean.ne[1] != c.latent_dim || mean.ne[2] != 1 || mean.ne[3] != 1 ||
            stddev.ne != mean.ne || hidden.ne[0] != c.cond_dim || hidden.ne[1] <= 0 || hidden.ne[1] > 128 ||
            hidden.ne[2] != 1 || hidden.ne[3] != 1)
            throw std::runtime_error("cache dimensions disagree with model/--frames: " + path.string());
        Sample s;
        s.name = path.filename().string();
        s.frames = (int)mean.ne[0];
        s.tokens = (int)hidden.ne[1];
        s.source_id = cache.string("ac.cache.source_id");
        if (cache.has("ac.cache.prompt")) s.caption = cache.string("ac.cache.prompt");
        s.empty = cache.boolean("ac.cache.empty_prompt");
        s.mean = cache.read_f32("mean");
        s.stddev = cache.read_f32("stddev");
        s.hidden = cache.read_f32("hidden");
        for (float v : s.stddev)
            if (v < 0) throw std::runtime_error("cache has invalid posterior stddev");
        s.edit_start = std::max(0.0f, t_min);
        if (cache.has("ac.cache.time_min")) {
            s.edit_start = cache.f32("ac.cache.time_min");
            if (!std::isfinite(s.edit_start) || s.edit_start < 0 || s.edit_start >= 1 ||
                (t_min >= 0 && std::fabs(t_min - s.edit_start) > 1e-6f))
                throw std::runtime_error("cache has invalid or mismatched minimum time");
        }
        if (bridge) {
            if (s.frames != frames) throw std::runtime_error("edit-bridge requires fixed cache windows");
            const auto& pivot = cache.get("edit_pivot");
            if (pivot.ne != mean.ne) throw std::runtime_error("edit pivot shape mismatch");
            s.pivot = cache.read_f32("edit_pivot");
            s.edit_start = cache.f32("ac.cache.edit_flowstep");
            if (!std::isfinite(s.edit_start) || s.edit_start < 0 || s.edit_start >= 1 ||
                (t_min >= 0 && std::fabs(t_min - s.edit_start) > 1e-6f) ||
                std::any_of(s.stddev.begin(), s.stddev.end(), [](float v) { return v != 0; }))
                throw std::runtime_error("edit cache needs a fixed target and matching valid pivot time");
        }
        max_tokens = std::max(max_tokens, s.tokens);
        out.push_back(std::move(s));
    }
    if (out.empty()) throw std::runtime_error("no cached .gguf samples in " + directory);
    return out;
}

void usage() {
    fprintf(stderr, "usage: mf-train --dit model.gguf --cache directory --out adapter.gguf [options]\n"
                    "  --prompt-pool JSON optional training-only pool for legacy caches\n"
                    "  --frames N        cached frames per example (default 50 = 2s)\n"
                    "  --steps N         optimizer steps (default 100)\n"
                    "  --rank N          LoRA rank (default 8)\n"
                    "  --alpha F         LoRA alpha (default rank)\n"
                    "  --adapter-type lora|dora-rows  adaptation formulation (default lora)\n"
                    "  --first-layer N   adapt attention from this layer through the last (default last)\n"
                    "  --lr F            Adam learning rate (default 0.0001)\n"
                    "  --seed N          RNG seed (default 1234)\n"
                    "  --cfg-dropout F   caption dropout probability (default 0.1)\n"
                    "  --objective flow-matching|edit-bridge  target/pairing (default flow-matching)\n"
                    "  --t-min F         minimum physical time (default cached minimum, otherwise 0)\n"
                    "  --t-sampling uniform|logit-normal  training time density (default uniform)\n"
                    "  --t-mean F        logit-normal Gaussian mean (default 0)\n"
                    "  --t-std F         logit-normal Gaussian stddev (default 1)\n"
                    "  --validation DIR  separate cached validation tracks\n"
                    "  --eval-samples N  fixed probe windows (default 4; 0 uses all)\n"
                    "  --eval-draws N    draws per probe window (default 1; >1 stratifies time)\n"
                    "  --checkpoint-every N  save and evaluate every N steps (default 0)\n"
                    "  --device gpu|gpu:N  CUDA device (default gpu = device 0; this build has no CPU path)\n"
                    "  --max-batch N     samples per device microbatch (default min(accumulation, 8))\n"
                    "  --device-sampling draw the posterior and noise on the GPU (Philox, per seed and window)\n"
                    "Exact resume via .state sidecars.\n");
}

// One drawn training / probe window, ready for the device.  With on-device sampling, clean and
// noise hold the window's posterior mean and stddev, and `window` numbers its device draws.
struct Draw {
    std::vector<float> clean, noise;
    const Sample* sample;
    float t;
    bool uncond;
    uint64_t window = 0;
};

// Device microbatches of drawn windows: submitted in draw order, losses returned in that order.
class Batcher {
public:
    Batcher(act_ctx* ctx, const act_model_desc& m, int frames, int tokens, int max_batch, bool bridge,
            bool device_sampling, uint64_t seed)
        : ctx_(ctx), m_(m), frames_(frames), tokens_(tokens), max_(max_batch), bridge_(bridge),
          device_(device_sampling), seed_(seed) {}

    void add(Draw d) {
        // one device batch numbers its windows consecutively
        if (device_ && !pending_.empty() && d.window != pending_.back().window + 1) flush();
        pending_.push_back(std::move(d));
        if ((int)pending_.size() == max_) flush();
    }
    // submits what is pending; returns every loss since the last take()
    std::vector<float> take() {
        flush();
        std::vector<float> out;
        out.swap(losses_);
        return out;
    }

private:
    void flush() {
        if (pending_.empty()) return;
        const int n = (int)pending_.size();
        const size_t nx = (size_t)m_.latent_dim * frames_, nh = (size_t)tokens_ * m_.cond_dim;
        std::vector<float> clean(n * nx), noise(n * nx), hidden(n * nh, 0.f), t(n), pivot, start;
        std::vector<int32_t> uncond(n), valid(n);
        if (bridge_) {
            pivot.resize(n * nx);
            start.resize(n);
        }
        for (int i = 0; i < n; ++i) {
            const Draw& d = pending_[i];
            std::copy(d.clean.begin(), d.clean.end(), clean.begin() + i * nx);
            std::copy(d.noise.begin(), d.noise.end(), noise.begin() + i * nx);
            std::copy(d.sample->hidden.begin(), d.sample->hidden.end(), hidden.begin() + i * nh);
            t[i] = d.t;
            uncond[i] = d.uncond ? 1 : 0;
            valid[i] = d.sample->tokens;
            if (bridge_) {
                std::copy(d.sample->pivot.begin(), d.sample->pivot.end(), pivot.begin() + i * nx);
                start[i] = d.sample->edit_start;
            }
        }
        act_mf_batch b{};
        b.n = n;
        b.clean = clean.data();
        b.noise = noise.data();
        b.hidden = hidden.data();
        b.t = t.data();
        b.unconditional = uncond.data();
        b.valid_tokens = valid.data();
        b.pivot = bridge_ ? pivot.data() : nullptr;
        b.edit_start = bridge_ ? start.data() : nullptr;
        if (device_) {
            b.noise = nullptr;
            b.stddev = noise.data();
            b.sample_seed = seed_;
            b.window0 = pending_[0].window;
        }
        std::vector<float> loss(n);
        actf::check(ctx_, act_mf_step(ctx_, &b, loss.data()), "training step");
        for (float l : loss) {
            if (!std::isfinite(l)) throw std::runtime_error("nonfinite training loss");
            losses_.push_back(l);
        }
        pending_.clear();
    }

    act_ctx* ctx_;
    act_model_desc m_;
    int frames_, tokens_, max_;
    bool bridge_, device_;
    uint64_t seed_;
    std::vector<Draw> pending_;
    std::vector<float> losses_;
};

}  // namespace

int main(int argc, char** argv) {
    act_ctx* ctx = nullptr;
    try {
        std::string prompt_pool;
        std::string dit_path, cache_path, out_path, validation_path, device = "gpu";
        int frames = 50, steps = 100, rank = 8, first_layer = -1, max_batch = 0;
        int eval_samples = 4, eval_draws = 1, checkpoint_every = 0;
        actf::TrainControls controls;
        uint32_t seed = 1234;
        float alpha = -1, lr = 1e-4f, dropout = 0.1f;
        std::string t_sampling = "uniform";
        float t_mean = 0, t_std = 1;
        std::string objective = "flow-matching";
        std::string adapter_type = "lora";
        float t_min = -1;
        bool device_sampling = false;
        for (int i = 1; i < argc; ++i) {
            std::string a = argv[i];
            auto next = [&]() -> std::string {
                if (++i >= argc) throw std::runtime_error(a + " needs a value");
                return argv[i];
            };
            if (controls.parse(a, next)) {
            } else if (a == "--prompt-pool") prompt_pool = next();
            else if (a == "--dit") dit_path = next();
            else if (a == "--cache") cache_path = next();
            else if (a == "--out") out_path = next();
            else if (a == "--validation") validation_path = next();
            else if (a == "--device") device = next();
            else if (a == "--frames") frames = std::stoi(next());
            else if (a == "--steps") steps = std::stoi(next());
            else if (a == "--rank") rank = std::stoi(next());
            else if (a == "--alpha") alpha = std::stof(next());
            else if (a == "--adapter-type") adapter_type = next();
            else if (a == "--first-layer") first_layer = std::stoi(next());
            else if (a == "--lr") lr = std::stof(next());
            else if (a == "--cfg-dropout") dropout = std::stof(next());
            else if (a == "--t-sampling") t_sampling = next();
            else if (a == "--t-mean") t_mean = std::stof(next());
            else if (a == "--t-std") t_std = std::stof(next());
            else if (a == "--objective") objective = next();
            else if (a == "--t-min") t_min = std::stof(next());
            else if (a == "--seed") seed = (uint32_t)std::stoul(next());
            else if (a == "--eval-samples") eval_samples = std::stoi(next());
            else if (a == "--eval-draws") eval_draws = std::stoi(next());
            else if (a == "--checkpoint-every") checkpoint_every = std::stoi(next());
            else if (a == "--max-batch") max_batch = std::stoi(next());
            else if (a == "--device-sampling") device_sampling = true;
            else if (a == "--help" || a == "-h") {
                usage();
                fprintf(stderr, "%s", actf::TrainControls::help());
                return 0;
            } else throw std::runtime_error("unknown argument: " + a);
        }
        controls.validate();
        if (dit_path.empty() || cache_path.empty() || out_path.empty()) {
            usage();
            return 2;
        }
        if (steps <= 0 || frames <= 0 || frames > 750 || rank <= 0 || eval_samples < 0 || eval_draws <= 0 ||
            checkpoint_every < 0 || !std::isfinite(lr) || lr <= 0 || !std::isfinite(dropout) || dropout < 0 ||
            dropout > 1 || !std::isfinite(t_min) || (t_min != -1 && (t_min < 0 || t_min >= 1)) || max_batch < 0 ||
            (objective != "flow-matching" && objective != "edit-bridge"))
            throw std::runtime_error("invalid training settings");
        if (adapter_type != "lora" && adapter_type != "dora-rows")
            throw std::runtime_error("invalid training dimensions or adapter configuration");
        if (device_sampling && objective == "edit-bridge")
            throw std::runtime_error("--device-sampling draws a posterior; edit-bridge caches have fixed targets");
        if (std::filesystem::exists(out_path)) throw std::runtime_error("output already exists: " + out_path);
        const actf::MfTimeSampler time_sampler(t_sampling, t_mean, t_std);
        if (alpha == -1) alpha = (float)rank;
        const int device_index = actf::parse_device(device);
        GgufReader model(dit_path);
        const DitShape shape = dit_config(model);
        const act_model_desc& config = shape.desc;
        if (first_layer == -1) first_layer = config.layers - 1;
        int max_tokens = 1;
        auto samples = read_samples(cache_path, model, config, frames, max_tokens, objective, t_min);
        std::vector<Sample> validation;
        if (!validation_path.empty())
            validation = read_samples(validation_path, model, config, frames, max_tokens, objective, t_min);
        std::set<std::string> training_sources;
        for (const auto& s : samples) training_sources.insert(s.source_id);
        for (const auto& s : validation)
            if (training_sources.count(s.source_id))
                throw std::runtime_error("source track appears in both training and validation");
        std::vector<std::string> captions;
        for (const auto& s : samples)
            if (!s.caption.empty()) captions.push_back(s.caption);
        if (!prompt_pool.empty()) captions = actf::read_prompt_pool(prompt_pool);
        auto save_pool = [&](const std::string& path) {
            if (!captions.empty())
                actf::write_prompt_pool(actf::prompt_pool_path(path), path, captions, training_sources.size());
        };
        if (rank > config.dim || !std::isfinite(alpha) || alpha <= 0 || first_layer < 0 || first_layer >= config.layers)
            throw std::runtime_error("invalid training dimensions or adapter configuration");

        // the device context: MfTrainGraph's constructor (src/mf/train.h:47-138)
        if (max_batch == 0) max_batch = std::min(controls.accumulation, 8);
        act_adapter_desc ad{};
        ad.type = adapter_type == "dora-rows" ? ACT_ADAPTER_DORA_ROWS : ACT_ADAPTER_LORA;
        ad.rank = rank;
        ad.alpha = alpha;
        ad.first_layer = first_layer;
        ad.targets = controls.feedforward ? ACT_TARGETS_REFERENCE_FFN : ACT_TARGETS_REFERENCE;
        ad.seed = seed;
        ad.max_batch = max_batch;
        ad.frames = frames;
        ad.tokens = max_tokens;
        ad.prefix_frames = 0;
        actf::check(nullptr, act_create(&ctx, device_index, &config, &ad), "act_create");
        for (const auto& t : model.tensors())
            if (t.name.rfind("dit.", 0) == 0)
                actf::check(ctx, act_bind_weight(ctx, t.name.c_str(), (int)t.type, t.data, t.bytes), "act_bind_weight");
        actf::check(ctx, act_finalize(ctx), "act_finalize");
        // exact resume and checkpoint invariance need bit-for-bit reproducible steps
        actf::check(ctx, act_set_deterministic(ctx, 1), "act_set_deterministic");
        fprintf(stderr, "[train] adapter type: %s\n", adapter_type.c_str());
        const bool bridge = objective == "edit-bridge";
        Batcher batcher(ctx, config, frames, max_tokens, max_batch, bridge, device_sampling, seed);

        std::mt19937 rng(seed);
        std::uniform_real_distribution<float> uniform(0, 1);
        std::vector<size_t> order(samples.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = i;
        // compute_sample's draws (tools/mf-train.cpp:250-270)
        auto draw_sample = [&](const Sample& s, std::mt19937& random, bool drop, float fixed_t, bool training,
                               uint64_t window) {
            std::normal_distribution<float> gaussian;
            const int crop = training && controls.random_crop
                                 ? std::uniform_int_distribution<int>(0, s.frames - frames)(random)
                                 : (s.frames - frames) / 2;
            Draw d;
            d.clean.resize((size_t)frames * config.latent_dim);
            d.noise.resize(d.clean.size());
            d.window = window;
            for (size_t i = 0; i < d.clean.size(); ++i) {
                const size_t at = (i / frames) * s.frames + crop + i % frames;
                if (device_sampling) {  // the device draws clean = mean + stddev * z and the noise
                    d.clean[i] = s.mean[at];
                    d.noise[i] = s.stddev[at];
                    continue;
                }
                d.clean[i] = s.mean[at] + s.stddev[at] * gaussian(random);
                d.noise[i] = gaussian(random);
            }
            const float u = fixed_t >= 0 ? fixed_t : training ? time_sampler.sample(random) : uniform(random);
            const float start = s.edit_start;
            d.t = start + (1 - start) * u;
            d.sample = &s;
            d.uncond = drop || s.empty;
            return d;
        };
        auto evaluate = [&]() {
            std::mt19937 eval_rng(seed + 1);
            double loss = 0;
            const auto& probes = validation.empty() ? samples : validation;
            const size_t count = eval_samples == 0 ? probes.size() : std::min<size_t>((size_t)eval_samples, probes.size());
            for (size_t i = 0; i < count; ++i)
                for (int draw = 0; draw < eval_draws; ++draw)  // probe windows number from 2^63 up
                    batcher.add(draw_sample(probes[i], eval_rng, controls.eval_null,
                                            eval_draws > 1 ? ((float)draw + 0.5f) / eval_draws : -1.0f, false,
                                            (1ull << 63) + i * eval_draws + draw));
            for (float l : batcher.take()) loss += l;
            // probes leave no gradient behind
            actf::check(ctx, act_zero_grads(ctx), "act_zero_grads");
            return loss / (count * eval_draws);
        };
        fprintf(stderr, "[train] probe: %d windows (0=all), %d draws per window\n", eval_samples, eval_draws);
        fprintf(stderr,
                "[train] training time density: %s (Gaussian mean %.4f, stddev %.4f); validation "
                "uniform/stratified\n",
                t_sampling.c_str(), t_mean, t_std);
        fprintf(stderr, "[train] objective %s; minimum physical time %s\n", objective.c_str(),
                t_min < 0 ? "from cache when present, otherwise 0" : std::to_string(t_min).c_str());
        fprintf(stderr, "[train] %zu training / %zu validation windows; fixed %s probe before %.7f\n", samples.size(),
                validation.size(), validation.empty() ? "training" : "validation", evaluate());
        std::string state_signature = controls.signature(lr) + actf::train_file_identity(dit_path) +
                                      actf::train_key(frames, rank, alpha, dropout, seed, objective, t_sampling, t_mean,
                                                      t_std, t_min, adapter_type, first_layer);
        if (device_sampling) state_signature += "|device-sampling";
        for (const auto& dir : {cache_path, validation_path})
            if (!dir.empty())
                for (const auto& p : actf::gguf_files(dir))
                    state_signature +=
                        "|" + std::filesystem::path(p).filename().string() + ":" + actf::train_file_identity(p);
        int completed = 0;
        size_t seen = 0;
        if (!controls.resume.empty()) {
            auto params = actf::read_params(ctx, true);
            actf::train_state(controls.resume, true, state_signature, params, completed, seen, rng, order);
            actf::write_params(ctx, params);
        }
        if (completed < 0 || completed >= steps || seen != (size_t)completed * controls.accumulation)
            throw std::runtime_error("invalid resume step/exposure or target steps");
        auto save_state = [&](const std::string& path) {
            auto params = actf::read_params(ctx, true);
            actf::train_state(path + ".state", false, state_signature, params, completed, seen, rng, order);
        };
        // MfTrainGraph::save (src/mf/train.h:229-255)
        auto save = [&](const std::string& path) {
            actf::save_adapter(ctx, path, [&](actf::GgufWriter& g) {
                g.add_string("general.architecture", "ac-melodyflow-lora");
                g.add_u32("ac.lora.version", 1);
                g.add_u32("ac.lora.rank", (uint32_t)rank);
                g.add_f32("ac.lora.alpha", alpha);
                g.add_string("ac.lora.type", adapter_type);
                g.add_string("ac.lora.training_activation", "erf-approx-as-7.1.26");
                g.add_string("ac.lora.training_objective", objective);
                g.add_string("ac.lora.training_time_density", t_sampling);
                if (!shape.name.empty()) g.add_string("ac.lora.base_name", shape.name);
            });
        };
        const auto start = std::chrono::steady_clock::now();
        for (int step = completed + 1; step <= steps; ++step) {
            for (int micro = 0; micro < controls.accumulation; ++micro) {
                const size_t index = seen % order.size();
                if (index == 0) std::shuffle(order.begin(), order.end(), rng);
                const auto& sample = samples[order[index]];
                const bool drop = uniform(rng) < dropout;
                batcher.add(draw_sample(sample, rng, drop, -1.f, true, seen));
                ++seen;
            }
            double loss = 0;
            for (float l : batcher.take()) loss += l;
            const float applied_lr = controls.rate(lr, step);
            // TrainAccumulation::update: mean over the microbatches, global clip, AdamW
            const act_opt o = controls.opt(applied_lr, step, controls.accumulation);
            int nonfinite = 0;
            const int rc = act_optimizer(ctx, &o, &nonfinite);
            if (rc == ACT_ERR_NONFINITE) throw std::runtime_error("nonfinite optimizer update");
            actf::check(ctx, rc, "act_optimizer");
            completed = step;
            fprintf(stderr, "[train] step %d/%d windows %zu lr %.9g loss %.7f\n", step, steps, seen, applied_lr,
                    loss / controls.accumulation);
            if (checkpoint_every > 0 && step % checkpoint_every == 0 && step < steps) {
                const auto output = std::filesystem::path(out_path);
                const auto checkpoint =
                    output.parent_path() / (output.stem().string() + ".step-" + std::to_string(step) + ".gguf");
                save(checkpoint.string());
                save_pool(checkpoint.string());
                save_state(checkpoint.string());
                fprintf(stderr, "[train] fixed probe step %d %.7f; saved %s\n", step, evaluate(),
                        checkpoint.string().c_str());
            }
        }
        fprintf(stderr, "[train] fixed probe after %.7f; %.2fs elapsed\n", evaluate(),
                std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count());
        save(out_path);
        save_pool(out_path);
        save_state(out_path);
        fprintf(stderr, "[train] saved %s\n", out_path.c_str());
        act_destroy(ctx);
        return 0;
    } catch (const std::exception& e) {
        fprintf(stderr, "error: %s\n", e.what());
        if (ctx) act_destroy(ctx);
        return 1;
    }
}
