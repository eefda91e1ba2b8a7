// mg-train on the B200 step: MusicGen LM adapter training (teacher-forced cross-entropy over the
// delay-pattern sequence) from cached codec tokens and projected conditioning.
//
// Same flags, sampling, accumulation, checkpoints, adapter file, caption pool, evaluation modes and
// exact-resume state as the reference front end (tools/mg-train.cpp:1-289); the forward/backward
// and AdamW run on the GPU through the act_* C ABI (the delay pattern and the selected rows are
// built by the library, src/mg/train.h:178-227).
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

struct LmShape {
    act_model_desc desc{};
    std::string name;
};

// LmConfig::from (src/mg/lm.h:60-90)
LmShape lm_config(const GgufReader& m) {
    if (m.string("ac.architecture") != "audiocraft") throw actf::GgufError("not an audiocraft GGUF");
    if (m.u32("ac.format_version") != 1) throw actf::GgufError("unsupported audiocraft GGUF version");
    if (m.string("ac.lm.family") != "musicgen") throw actf::GgufError("not a MusicGen LM GGUF");
    LmShape s;
    auto& d = s.desc;
    d.family = ACT_FAMILY_MUSICGEN;
    d.dim = (int)m.u32("ac.lm.dim");
    d.layers = (int)m.u32("ac.lm.layers");
    d.heads = (int)m.u32("ac.lm.heads");
    d.head_dim = (int)m.u32("ac.lm.head_dim");
    d.ff_dim = (int)m.u32("ac.lm.ff_dim");
    (void)m.u32("ac.lm.cond_dim");  // the caches hold conditioning already projected to dim
    d.n_q = (int)m.u32("ac.lm.n_q");
    d.card = (int)m.u32("ac.lm.card");
    d.special_token_id = (int)m.u32("ac.lm.special_token_id");
    d.pos_denominator = (int)m.u32("ac.lm.pos_denominator");
    d.max_period = m.f32("ac.lm.max_period");
    d.norm_eps = m.f32("ac.lm.norm_eps");
    (void)m.f32("ac.lm.cfg_coef");
    (void)m.u32("ac.lm.sample_rate");
    (void)m.f32("ac.lm.max_duration");
    if (d.dim != d.heads * d.head_dim) throw actf::GgufError("LM dim does not equal heads * head_dim");
    if (d.special_token_id != d.card)
        throw actf::GgufError("special_token_id should be card: it is the extra embedding row");
    if (m.has("general.name")) s.name = m.string("general.name");
    return s;
}

struct Sample {
    std::string name, source, caption;
    std::vector<int32_t> codes;  // [n_q][frames]
    std::vector<float> context;  // [tokens][dim]
    int tokens = 0, frames = 0;
};

// read_samples (tools/mg-train.cpp:14-62)
std::vector<Sample> read_samples(const std::string& dir, const LmShape& model, int frames, int& tokens) {
    const auto& c = model.desc;
    std::vector<Sample> out;
    for (const auto& file : actf::gguf_files(dir)) {
        GgufReader cache(file);
        if (cache.string("general.architecture") != "ac-musicgen-train-cache" || cache.u32("ac.cache.version") != 1 ||
            cache.string("ac.cache.base_name") != model.name)
            throw std::runtime_error("cache/base mismatch: " + file);
        const auto& codes = cache.get("codes");
        const auto& context = cache.get("context");
        if (codes.type != actf::GT_I32 || codes.ne[0] < frames || codes.ne[1] != c.n_q || codes.ne[2] != 1 ||
            codes.ne[3] != 1 || context.type != actf::GT_F32 || context.ne[0] != c.dim || context.ne[1] <= 0 ||
            context.ne[1] > 128 || context.ne[2] != 1 || context.ne[3] != 1)
            throw std::runtime_error("invalid training cache dimensions");
        Sample s;
        s.name = std::filesystem::path(file).filename().string();
        s.frames = (int)codes.ne[0];
        s.source = cache.string("ac.cache.source_id");
        if (s.source.empty()) throw std::runtime_error("cache source_id must not be empty");
        s.caption = cache.string("ac.cache.prompt");
        s.codes.assign(reinterpret_cast<const int32_t*>(codes.data),
                       reinterpret_cast<const int32_t*>(codes.data) + codes.nelements());
        for (auto v : s.codes)
            if (v < 0 || v >= c.card) throw std::runtime_error("invalid codec token");
        s.context = cache.read_f32("context");
        s.tokens = (int)context.ne[1];
        tokens = std::max(tokens, s.tokens);
        out.push_back(std::move(s));
    }
    if (out.empty()) throw std::runtime_error("no cached samples in " + dir);
    return out;
}

// Device microbatches of windows, submitted in order; losses come back in that order.
class Batcher {
public:
    Batcher(act_ctx* ctx, const act_model_desc& m, int frames, int tokens, int max_batch)
        : ctx_(ctx), m_(m), frames_(frames), tokens_(tokens), max_(max_batch) {}

    // compute()'s inputs (tools/mg-train.cpp:176-188): context padded to the longest cache (zeros
    // for a dropped caption), codes cropped to the window
    void add(const Sample& s, bool drop, int crop) {
        const size_t nc = (size_t)frames_ * m_.n_q, nx = (size_t)tokens_ * m_.dim;
        codes_.resize(codes_.size() + nc);
        int32_t* dst = codes_.data() + codes_.size() - nc;
        for (int q = 0; q < m_.n_q; ++q)
            std::copy_n(s.codes.begin() + (size_t)q * s.frames + crop, frames_, dst + (size_t)q * frames_);
        context_.resize(context_.size() + nx, 0.f);
        if (!drop) std::copy(s.context.begin(), s.context.end(), context_.end() - nx);
        if (++n_ == max_) flush();
    }
    std::vector<float> take() {
        flush();
        std::vector<float> out;
        out.swap(losses_);
        return out;
    }

private:
    void flush() {
        if (!n_) return;
        act_mg_batch b{};
        b.n = n_;
        b.codes = codes_.data();
        b.context = context_.data();
        std::vector<float> loss(n_);
        actf::check(ctx_, act_mg_step(ctx_, &b, loss.data()), "training step");
        for (float l : loss) {
            if (!std::isfinite(l)) throw std::runtime_error("nonfinite training loss");
            losses_.push_back(l);
        }
        n_ = 0;
        codes_.clear();
        context_.clear();
    }

    act_ctx* ctx_;
    act_model_desc m_;
    int frames_, tokens_, max_, n_ = 0;
    std::vector<int32_t> codes_;
    std::vector<float> context_;
    std::vector<float> losses_;
};

void help() {
    fprintf(stderr,
            "usage: mg-train --lm model.gguf --cache DIR --out adapter.gguf\n"
            "  --validation DIR --frames 600 --prefix-frames 0 (full-sequence loss; >0 masks a "
            "prefix) --steps 500 --rank 32\n"
            "  --alpha RANK --first-layer N (default last 12) --adapter-type dora-rows|lora\n"
            "  --lr 0.0001 --cfg-dropout 0.1 --seed 1234 --device gpu|gpu:N\n"
            "  --checkpoint-every 250 --eval-samples 8 (0=all) --max-batch N (default min(accumulation, 8))\n"
            "  --evaluate-only or --evaluate-adapter FILE  score without training/writing\n"
            "Teacher-forced cross-entropy; prefix/special tokens excluded; exact resume via "
            ".state sidecars.\n");
}

}  // namespace

int main(int argc, char** argv) {
    act_ctx* ctx = nullptr;
    try {
        std::string lm_path, cache_path, out_path, validation_path, device = "gpu", type = "dora-rows",
                                                                    evaluate_adapter;
        bool evaluate_only = false;
        int frames = 600, prefix = 0, steps = 500, rank = 32, first = -1, checkpoint = 250, eval_samples = 8;
        int max_batch = 0;
        float alpha = -1, lr = 1e-4f, dropout = 0.1f;
        actf::TrainControls controls;
        uint32_t seed = 1234;
        for (int i = 1; i < argc; ++i) {
            std::string a = argv[i];
            auto next = [&]() {
                if (++i >= argc) throw std::runtime_error(a + " needs a value");
                return std::string(argv[i]);
            };
            if (controls.parse(a, next)) {
            } else if (a == "--lm") lm_path = next();
            else if (a == "--cache") cache_path = next();
            else if (a == "--out") out_path = next();
            else if (a == "--validation") validation_path = next();
            else if (a == "--device") device = next();
            else if (a == "--adapter-type") type = next();
            else if (a == "--evaluate-only") evaluate_only = true;
            else if (a == "--evaluate-adapter") {
                evaluate_adapter = next();
                evaluate_only = true;
            } else if (a == "--frames") frames = std::stoi(next());
            else if (a == "--prefix-frames") prefix = std::stoi(next());
            else if (a == "--steps") steps = std::stoi(next());
            else if (a == "--rank") rank = std::stoi(next());
            else if (a == "--first-layer") first = std::stoi(next());
            else if (a == "--checkpoint-every") checkpoint = std::stoi(next());
            else if (a == "--eval-samples") eval_samples = std::stoi(next());
            else if (a == "--alpha") alpha = std::stof(next());
            else if (a == "--lr") lr = std::stof(next());
            else if (a == "--cfg-dropout") dropout = std::stof(next());
            else if (a == "--seed") seed = (uint32_t)std::stoul(next());
            else if (a == "--max-batch") max_batch = std::stoi(next());
            else if (a == "--help" || a == "-h") {
                help();
                fprintf(stderr, "%s", actf::TrainControls::help());
                return 0;
            } else throw std::runtime_error("unknown option: " + a);
        }
        controls.validate();
        if (lm_path.empty() || cache_path.empty() || (!evaluate_only && out_path.empty()) || steps <= 0 ||
            checkpoint < 0 || eval_samples < 0 || !std::isfinite(dropout) || dropout < 0 || dropout > 1 ||
            !std::isfinite(lr) || lr <= 0 || max_batch < 0)
            throw std::runtime_error("missing required paths or invalid training options");
        if (alpha == -1) alpha = (float)rank;
        if (!evaluate_only &&
            (std::filesystem::exists(out_path) || std::filesystem::exists(actf::prompt_pool_path(out_path))))
            throw std::runtime_error("output already exists");
        const int device_index = actf::parse_device(device);
        GgufReader model(lm_path);
        const LmShape shape = lm_config(model);
        const act_model_desc& config = shape.desc;
        if (first == -1) first = std::max(0, config.layers - 12);
        int tokens = 0;
        auto samples = read_samples(cache_path, shape, frames, tokens);
        std::vector<Sample> validation;
        if (!validation_path.empty()) validation = read_samples(validation_path, shape, frames, tokens);
        std::set<std::string> sources;
        for (const auto& s : samples) sources.insert(s.source);
        for (const auto& s : validation)
            if (sources.count(s.source)) throw std::runtime_error("training/validation track overlap");
        std::vector<std::string> captions;
        for (const auto& s : samples) captions.push_back(s.caption);
        if (std::all_of(captions.begin(), captions.end(), [](const std::string& s) { return s.empty(); }))
            throw std::runtime_error("no training captions for prompt pool");
        // MgTrainGraph's constructor checks (src/mg/train.h:66-73)
        if (frames <= 0 || tokens <= 0 || prefix < 0 || prefix >= frames || rank <= 0 || rank > config.dim ||
            !std::isfinite(alpha) || alpha <= 0 || first < 0 || first >= config.layers ||
            (type != "lora" && type != "dora-rows"))
            throw std::runtime_error("invalid MusicGen training configuration");

        if (max_batch == 0) max_batch = std::min(controls.accumulation, 8);
        act_adapter_desc ad{};
        ad.type = type == "dora-rows" ? ACT_ADAPTER_DORA_ROWS : ACT_ADAPTER_LORA;
        ad.rank = rank;
        ad.alpha = alpha;
        ad.first_layer = first;
        ad.targets = controls.feedforward ? ACT_TARGETS_REFERENCE_FFN : ACT_TARGETS_REFERENCE;
        ad.seed = seed;
        ad.max_batch = max_batch;
        ad.frames = frames;
        ad.tokens = tokens;
        ad.prefix_frames = prefix;
        actf::check(nullptr, act_create(&ctx, device_index, &config, &ad), "act_create");
        for (const auto& t : model.tensors())
            if (t.name.rfind("lm.", 0) == 0)
                actf::check(ctx, act_bind_weight(ctx, t.name.c_str(), (int)t.type, t.data, t.bytes), "act_bind_weight");
        actf::check(ctx, act_finalize(ctx), "act_finalize");
        // exact resume and checkpoint invariance need bit-for-bit reproducible steps
        actf::check(ctx, act_set_deterministic(ctx, 1), "act_set_deterministic");
        if (!evaluate_adapter.empty()) {
            // the adapter must adapt exactly this configuration (load_mg_lora, src/ac/lora.h:178-210)
            GgufReader adapter(evaluate_adapter);
            auto params = actf::read_params(ctx, false);
            const auto map = actf::load_lora(model, adapter, 1.0f, "lm");
            const size_t per = type == "dora-rows" ? 3 : 2;
            if (map.size() * per != params.size() || adapter.f32("ac.lora.alpha") != alpha ||
                adapter.string("ac.lora.type") != type)
                throw std::runtime_error("evaluation adapter configuration mismatch");
            for (auto& p : params) {
                const auto& t = adapter.get(p.name);
                if (t.type != actf::GT_F32 || t.ne[0] != p.cols || t.ne[1] != p.rows || t.ne[2] != 1 || t.ne[3] != 1)
                    throw std::runtime_error("evaluation adapter shape mismatch");
                p.value = adapter.read_f32(p.name);
            }
            actf::write_params(ctx, params);
        }
        Batcher batcher(ctx, config, frames, tokens, max_batch);
        auto evaluate = [&]() {
            const auto& probes = validation.empty() ? samples : validation;
            const size_t n = eval_samples == 0 ? probes.size() : std::min(probes.size(), (size_t)eval_samples);
            double sum = 0;
            for (size_t i = 0; i < n; ++i) batcher.add(probes[i], controls.eval_null, (probes[i].frames - frames) / 2);
            for (float l : batcher.take()) sum += l;
            actf::check(ctx, act_zero_grads(ctx), "act_zero_grads");  // probes leave no gradient behind
            return sum / n;
        };
        if (evaluate_only) {
            fprintf(stderr, "[eval] %s prefix %d fixed probe %.7f\n",
                    evaluate_adapter.empty() ? "base" : evaluate_adapter.c_str(), prefix, evaluate());
            act_destroy(ctx);
            return 0;
        }
        // MgTrainGraph::save (src/mg/train.h:255-289) and the caption pool beside it
        auto save = [&](const std::string& path) {
            if (std::filesystem::exists(actf::prompt_pool_path(path))) throw std::runtime_error("prompt pool already exists");
            actf::save_adapter(ctx, path, [&](actf::GgufWriter& g) {
                g.add_string("general.architecture", "ac-musicgen-lora");
                g.add_u32("ac.lora.version", 1);
                g.add_u32("ac.lora.rank", (uint32_t)rank);
                g.add_f32("ac.lora.alpha", alpha);
                g.add_string("ac.lora.type", type);
                g.add_string("ac.lora.training_activation", "erf-approx-as-7.1.26");
                g.add_string("ac.lora.training_objective",
                             prefix == 0 ? "generation-cross-entropy" : "continuation-cross-entropy");
                g.add_u32("ac.lora.training_frames", (uint32_t)frames);
                g.add_u32("ac.lora.prefix_frames", (uint32_t)prefix);
                if (!shape.name.empty()) g.add_string("ac.lora.base_name", shape.name);
            });
            actf::write_prompt_pool(actf::prompt_pool_path(path), path, captions, sources.size());
        };
        fprintf(stderr,
                "[train] %zu training / %zu validation windows; %d prefix, %d continuation frames; fixed "
                "probe before %.7f\n",
                samples.size(), validation.size(), prefix, frames - prefix, evaluate());
        std::mt19937 rng(seed);
        std::uniform_real_distribution<float> uniform(0, 1);
        std::vector<size_t> order(samples.size());
        for (size_t i = 0; i < order.size(); ++i) order[i] = i;
        std::string state_signature = controls.signature(lr) + actf::train_file_identity(lm_path) +
                                      actf::train_key(frames, rank, alpha, dropout, seed, prefix, type, first);
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
        const auto start = std::chrono::steady_clock::now();
        for (int step = completed + 1; step <= steps; ++step) {
            for (int micro = 0; micro < controls.accumulation; ++micro) {
                const size_t index = seen % order.size();
                if (index == 0) std::shuffle(order.begin(), order.end(), rng);
                const auto& sample = samples[order[index]];
                const bool drop = uniform(rng) < dropout;
                const int crop = controls.random_crop ? std::uniform_int_distribution<int>(0, sample.frames - frames)(rng)
                                                      : (sample.frames - frames) / 2;
                batcher.add(sample, drop, crop);
                ++seen;
            }
            double loss = 0;
            for (float l : batcher.take()) loss += l;
            const float applied_lr = controls.rate(lr, step);
            const act_opt o = controls.opt(applied_lr, step, controls.accumulation);
            int nonfinite = 0;
            const int rc = act_optimizer(ctx, &o, &nonfinite);
            if (rc == ACT_ERR_NONFINITE) throw std::runtime_error("nonfinite optimizer update");
            actf::check(ctx, rc, "act_optimizer");
            completed = step;
            fprintf(stderr, "[train] step %d/%d windows %zu lr %.9g loss %.7f\n", step, steps, seen, applied_lr,
                    loss / controls.accumulation);
            if (checkpoint > 0 && step % checkpoint == 0 && step < steps) {
                const auto p = std::filesystem::path(out_path);
                const auto path = (p.parent_path() / (p.stem().string() + ".step-" + std::to_string(step) + ".gguf")).string();
                save(path);
                save_state(path);
                fprintf(stderr, "[train] fixed probe step %d %.7f\n", step, evaluate());
            }
        }
        fprintf(stderr, "[train] fixed probe after %.7f; %.2fs elapsed\n", evaluate(),
                std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count());
        save(out_path);
        save_state(out_path);
        act_destroy(ctx);
        return 0;
    } catch (const std::exception& e) {
        fprintf(stderr, "error: %s\n", e.what());
        if (ctx) act_destroy(ctx);
        return 1;
    }
}
