"""Files and a replay for the trainer front-end tests.

write_dit / write_caches make a tiny MelodyFlow DiT GGUF and training (or edit-bridge) caches with
the metadata mf-train reads (src/mf/dit.h:44-71, tools/mf-train.cpp:17-95).  MfTrainReplay redoes
mf-train's loop in Python: the same standard-library draws (stdrng) in the same order, the step and
AdamW of the CPU oracle, so the losses mf-train prints can be checked against the oracle.
"""
import os

import numpy as np

import oracle as O
import stdrng as R

F32 = np.float32


def _gguf():
    import gguf
    return gguf


def write_gguf(path, arch, tensors, metadata):
    gguf = _gguf()
    w = gguf.GGUFWriter(str(path), arch)
    for key, value in metadata.items():
        if isinstance(value, bool):
            w.add_bool(key, value)
        elif isinstance(value, int):
            w.add_uint32(key, value)
        elif isinstance(value, float):
            w.add_float32(key, value)
        else:
            w.add_string(key, value)
    for key, value in tensors.items():
        w.add_tensor(key, np.ascontiguousarray(value))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


class TinyDit:
    """A DiT our kernels run (head_dim 64) and the oracle's weights for it."""

    def __init__(self, dim=128, layers=4, heads=2, ff=256, lat=32, cond=32, tdim=16, seed=3, wstd=0.05):
        self.cfg = O.DitCfg(dim, layers, heads, dim // heads, ff, lat, cond, tdim, (layers - 1) // 2, 1e-5, 1)
        rng = np.random.default_rng(seed)
        self.names = O.dit_tensor_names(self.cfg)
        shapes = O.dit_tensor_shapes(self.cfg)
        W = {}
        for n, (r, c) in zip(self.names, shapes):
            if n.endswith("rope_freq_factors"):
                w = (10000.0 ** (2 * np.arange(c) / 64.0)).astype(F32)
            elif "norm" in n and n.endswith(".weight"):
                w = (1.0 + 0.1 * rng.standard_normal(c)).astype(F32)
            elif "norm" in n or n.endswith(".bias"):
                w = (0.05 * rng.standard_normal(c)).astype(F32)
            else:
                w = (wstd * rng.standard_normal((r, c) if r > 1 else c)).astype(F32)
            W[n] = w
        self.W = W
        self.Wflat = np.concatenate([W[n].ravel() for n in self.names]).astype(F32)
        self.latent_mean = (0.1 * rng.standard_normal(lat)).astype(F32)
        self.latent_std = (1.0 + 0.1 * rng.random(lat)).astype(F32)

    def write(self, path, name="tiny test dit"):
        c = self.cfg
        meta = {"general.name": name, "ac.architecture": "audiocraft", "ac.format_version": 1,
                "ac.dit.family": "melodyflow", "ac.dit.dim": c.dim, "ac.dit.layers": c.layers,
                "ac.dit.heads": c.heads, "ac.dit.head_dim": c.head_dim, "ac.dit.ff_dim": c.ff_dim,
                "ac.dit.latent_dim": c.latent_dim, "ac.dit.cond_dim": c.cond_dim, "ac.dit.time_dim": c.time_dim,
                "ac.dit.n_skip": c.n_skip, "ac.dit.rope_base": 10000.0, "ac.dit.norm_eps": 1e-5,
                "ac.dit.cfg_coef": 4.0, "ac.dit.max_duration": 30.0, "ac.dit.add_zero_attn": True}
        tensors = dict(self.W)
        tensors["dit.latent_mean"] = self.latent_mean
        tensors["dit.latent_std"] = self.latent_std
        write_gguf(path, "audiocraft", tensors, meta)

    def norm_std(self):
        return (self.latent_std + F32(1e-5)).astype(F32)


def write_caches(directory, dit, n, frames, seed, tokens=(5, 8), empty=(), captions=None, bridge_start=None,
                 prefix="sample"):
    """n cache files; with bridge_start, edit-bridge caches (fixed target, pivot, flow step)."""
    os.makedirs(directory, exist_ok=True)
    rng = np.random.default_rng(seed)
    lat, cond = dit.cfg.latent_dim, dit.cfg.cond_dim
    for i in range(n):
        ntok = tokens[i % len(tokens)]
        mean = rng.normal(0, 0.5, (lat, frames)).astype(F32)
        std = (np.zeros if bridge_start is not None else lambda s: rng.uniform(0.05, 0.3, s))((lat, frames)).astype(F32)
        t = {"mean": mean, "stddev": std, "hidden": rng.normal(0, 0.5, (ntok, cond)).astype(F32),
             "normalization_mean": dit.latent_mean, "normalization_std": dit.norm_std()}
        meta = {"ac.cache.version": 1, "ac.cache.empty_prompt": i in empty,
                "ac.cache.source_id": f"{os.path.basename(directory)}-{prefix}-{i}"}
        if captions:
            meta["ac.cache.prompt"] = captions[i % len(captions)]
        arch = "ac-melodyflow-train-cache"
        if bridge_start is not None:
            arch = "ac-melodyflow-edit-cache"
            t["edit_pivot"] = (mean + rng.normal(0, 0.5, mean.shape)).astype(F32)
            meta["ac.cache.edit_flowstep"] = float(bridge_start)
        write_gguf(os.path.join(directory, f"{prefix}-{i}.gguf"), arch, t, meta)


def read_caches(directory):
    gguf = _gguf()
    out = []
    for f in sorted(p for p in os.listdir(directory) if p.endswith(".gguf")):
        r = gguf.GGUFReader(os.path.join(directory, f))
        t = {x.name: np.array(x.data) for x in r.tensors}
        fields = {k: v.contents() for k, v in r.fields.items() if not k.startswith("GGUF.")}
        s = {"mean": t["mean"].astype(F32).ravel(), "stddev": t["stddev"].astype(F32).ravel(),
             "frames": t["mean"].shape[-1], "hidden": t["hidden"].astype(F32), "tokens": t["hidden"].shape[0],
             "empty": bool(fields["ac.cache.empty_prompt"]), "start": 0.0}
        if "edit_pivot" in t:
            s["pivot"] = t["edit_pivot"].astype(F32).ravel()
            s["start"] = F32(fields["ac.cache.edit_flowstep"])
        out.append(s)
        del r
    return out


def read_adapter(path):
    gguf = _gguf()
    r = gguf.GGUFReader(str(path))
    out = {t.name: np.array(t.data, dtype=F32).ravel() for t in r.tensors}
    meta = {k: v.contents() for k, v in r.fields.items() if not k.startswith("GGUF.")}
    del r
    return out, meta


class MfTrainReplay:
    """mf-train's loop (tools/mf-train.cpp:230-346) on the CPU oracle, LoRA adapters."""

    def __init__(self, dit, train, validation, frames, rank, alpha, first_layer, seed, targets, accumulation=1,
                 dropout=0.1, random_crop=False, t_sampling="uniform", t_mean=0.0, t_std=1.0, eval_samples=4,
                 eval_draws=1, eval_null=False, lr=1e-4, warmup=0, schedule="constant", beta1=0.9, beta2=0.999,
                 eps=1e-8, decay=0.0, clip=1.0, bridge=False):
        self.__dict__.update({k: v for k, v in locals().items() if k not in ("self", "train", "validation")})
        self.samples, self.probes_ = train, validation
        self.ad = O.Adapter(rank, alpha, 0, first_layer, targets)
        self.layout = O.adapter_layout(dit.cfg.dim, dit.cfg.ff_dim, dit.cfg.layers, self.ad)
        self.max_tokens = max(s["tokens"] for s in train + validation)
        # MfTrainGraph's initialisation: lora_A ~ N(0, 0.02) from mt19937(seed) in parameter order
        # (one distribution for all tensors), lora_B = 0 (src/mf/train.h:65-101)
        g, normal = R.MT19937(seed), R.Normal(0.0, 0.02)
        n = sum(int(np.prod(shape)) for _, _, shape in self.layout)
        self.params = np.zeros(n, F32)
        self.decay_mask = np.zeros(n, np.uint8)
        for name, off, shape in self.layout:
            k = int(np.prod(shape))
            if name.endswith("lora_A"):
                self.params[off:off + k] = [normal(g) for _ in range(k)]
            if name.endswith(("lora_A", "lora_B")):
                self.decay_mask[off:off + k] = 1
        self.m = np.zeros(n, F32)
        self.v = np.zeros(n, F32)

    def draw(self, s, g, drop, fixed_t, training):
        gauss = R.Normal()
        frames, lat = self.frames, self.dit.cfg.latent_dim
        crop = R.uniform_int(g, 0, s["frames"] - frames) if training and self.random_crop else (s["frames"] - frames) // 2
        clean = np.empty(frames * lat, F32)
        noise = np.empty(frames * lat, F32)
        for i in range(frames * lat):
            at = (i // frames) * s["frames"] + crop + i % frames
            clean[i] = s["mean"][at] + s["stddev"][at] * gauss(g)
            noise[i] = gauss(g)
        if fixed_t >= 0:
            u = F32(fixed_t)
        elif training:
            u = R.time_sample(g, self.t_sampling, self.t_mean, self.t_std)
        else:
            u = R.uniform_real(g)
        start = F32(s["start"])
        t = start + (F32(1) - start) * u
        if self.bridge:  # compute_bridge's endpoint (src/mf/train.h:196-203)
            noise = ((s["pivot"] - start * clean) / (F32(1) - start)).astype(F32)
        return clean, noise, t, drop or s["empty"], s

    def _run(self, draws, grads):
        lat, cond, frames = self.dit.cfg.latent_dim, self.dit.cfg.cond_dim, self.frames
        n = len(draws)
        clean = np.stack([d[0] for d in draws]).reshape(n, lat, frames)
        noise = np.stack([d[1] for d in draws]).reshape(n, lat, frames)
        hidden = np.zeros((n, self.max_tokens, cond), F32)
        for i, d in enumerate(draws):
            hidden[i, :d[4]["tokens"]] = d[4]["hidden"]
        t = np.array([d[2] for d in draws], F32)
        unc = np.array([int(d[3]) for d in draws], np.int32)
        valid = np.array([d[4]["tokens"] for d in draws], np.int32)
        return O.dit_step(self.dit.cfg, self.dit.Wflat, self.ad, self.params, clean, noise, hidden, t, unc, valid,
                          grads=grads)

    def evaluate(self):
        g = R.MT19937(self.seed + 1)
        probes = self.probes_ or self.samples
        count = len(probes) if self.eval_samples == 0 else min(self.eval_samples, len(probes))
        draws = []
        for i in range(count):
            for d in range(self.eval_draws):
                fixed = (d + 0.5) / self.eval_draws if self.eval_draws > 1 else -1.0
                draws.append(self.draw(probes[i], g, self.eval_null, np.float32(fixed) if fixed >= 0 else -1.0, False))
        loss, _ = self._run(draws, False)
        return float(np.sum(loss.astype(np.float64))) / (count * self.eval_draws)

    def rate(self, step):
        factor = min(F32(1), F32(step) / F32(self.warmup)) if self.warmup else F32(1)
        if self.schedule == "inverse":
            factor = F32(factor * F32(np.power(F32(1) + F32(step - 1) / F32(1e6), F32(-0.5))))
        return F32(F32(self.lr) * factor)

    def train(self, steps):
        """Per-step mean losses (and the probe before), as mf-train prints them."""
        g = R.MT19937(self.seed)
        order = list(range(len(self.samples)))
        seen = 0
        out = {"before": self.evaluate(), "steps": []}
        for step in range(1, steps + 1):
            draws = []
            for _ in range(self.accumulation):
                index = seen % len(order)
                if index == 0:
                    R.shuffle(order, g)
                drop = R.uniform_real(g) < F32(self.dropout)
                draws.append(self.draw(self.samples[order[index]], g, drop, -1.0, True))
                seen += 1
            loss, grad = self._run(draws, True)
            out["steps"].append(float(np.sum(loss.astype(np.float64))) / self.accumulation)
            lr = O.lib().ora_rate(F32(self.lr), step, self.warmup, int(self.schedule == "inverse"))
            O.lib().ora_adamw(self.params.size, self.params, self.m, self.v, grad.astype(F32), self.decay_mask,
                              self.accumulation, step, lr, self.beta1, self.beta2, self.eps, self.decay, self.clip)
        out["after"] = self.evaluate()
        return out


# ----------------------------------------------------------------------------- MusicGen
class TinyLm:
    """A MusicGen LM our kernels run (head_dim 64) and the oracle's weights for it."""

    def __init__(self, dim=128, layers=2, heads=2, ff=256, n_q=4, card=64, seed=4, wstd=0.05):
        self.cfg = O.LmCfg(dim, layers, heads, dim // heads, ff, n_q, card, card, dim // 2 - 1, 10000.0, 1e-5)
        rng = np.random.default_rng(seed)
        self.names = O.lm_tensor_names(self.cfg)
        shapes = O.lm_tensor_shapes(self.cfg)
        W = {}
        for n, (r, c) in zip(self.names, shapes):
            if "norm" in n and n.endswith(".weight"):
                w = (1.0 + 0.1 * rng.standard_normal(c)).astype(F32)
            elif "norm" in n or n.endswith(".bias"):
                w = (0.05 * rng.standard_normal(c)).astype(F32)
            elif ".emb." in n:
                w = (0.5 * rng.standard_normal((r, c))).astype(F32)
            else:
                w = (wstd * rng.standard_normal((r, c) if r > 1 else c)).astype(F32)
            W[n] = w
        self.W = W
        self.Wflat = np.concatenate([W[n].ravel() for n in self.names]).astype(F32)
        self.name = "tiny test lm"

    def write(self, path):
        c = self.cfg
        meta = {"general.name": self.name, "ac.architecture": "audiocraft", "ac.format_version": 1,
                "ac.lm.family": "musicgen", "ac.lm.dim": c.dim, "ac.lm.layers": c.layers, "ac.lm.heads": c.heads,
                "ac.lm.head_dim": c.head_dim, "ac.lm.ff_dim": c.ff_dim, "ac.lm.cond_dim": 48, "ac.lm.n_q": c.n_q,
                "ac.lm.card": c.card, "ac.lm.special_token_id": c.card, "ac.lm.pos_denominator": c.dim // 2 - 1,
                "ac.lm.max_period": 10000.0, "ac.lm.norm_eps": 1e-5, "ac.lm.cfg_coef": 3.0,
                "ac.lm.sample_rate": 32000, "ac.lm.max_duration": 30.0}
        write_gguf(path, "ac-musicgen-lm", self.W, meta)


def write_mg_caches(directory, lm, n, frames, seed, tokens=(3, 6), caption="glitch hop, 92 bpm, D minor"):
    os.makedirs(directory, exist_ok=True)
    rng = np.random.default_rng(seed)
    for i in range(n):
        t = {"codes": rng.integers(0, lm.cfg.card, (lm.cfg.n_q, frames), dtype=np.int32),
             "context": rng.normal(0, 0.5, (tokens[i % len(tokens)], lm.cfg.dim)).astype(F32)}
        meta = {"ac.cache.version": 1, "ac.cache.base_name": lm.name,
                "ac.cache.source_id": f"{os.path.basename(directory)}-{i}", "ac.cache.prompt": caption}
        write_gguf(os.path.join(directory, f"{i}.gguf"), "ac-musicgen-train-cache", t, meta)


def read_mg_caches(directory):
    gguf = _gguf()
    out = []
    for f in sorted(p for p in os.listdir(directory) if p.endswith(".gguf")):
        r = gguf.GGUFReader(os.path.join(directory, f))
        t = {x.name: np.array(x.data) for x in r.tensors}
        out.append({"codes": t["codes"].astype(np.int32), "context": t["context"].astype(F32),
                    "frames": t["codes"].shape[-1], "tokens": t["context"].shape[0]})
        del r
    return out


class MgTrainReplay:
    """mg-train's loop (tools/mg-train.cpp:224-283) on the CPU oracle, LoRA adapters."""

    def __init__(self, lm, train, validation, frames, prefix, rank, alpha, first_layer, seed, targets,
                 accumulation=1, dropout=0.1, random_crop=False, eval_samples=8, eval_null=False, lr=1e-4, warmup=0,
                 schedule="constant", beta1=0.9, beta2=0.999, eps=1e-8, decay=0.0, clip=1.0):
        self.__dict__.update({k: v for k, v in locals().items() if k not in ("self", "train", "validation")})
        self.samples, self.probes_ = train, validation
        self.ad = O.Adapter(rank, alpha, 0, first_layer, targets)
        self.layout = O.adapter_layout(lm.cfg.dim, lm.cfg.ff_dim, lm.cfg.layers, self.ad, prefix="lm")
        self.tokens = max(s["tokens"] for s in train + validation)
        g, normal = R.MT19937(seed), R.Normal(0.0, 0.02)
        n = sum(int(np.prod(shape)) for _, _, shape in self.layout)
        self.params = np.zeros(n, F32)
        self.decay_mask = np.zeros(n, np.uint8)
        for name, off, shape in self.layout:
            k = int(np.prod(shape))
            if name.endswith("lora_A"):
                self.params[off:off + k] = [normal(g) for _ in range(k)]
            if name.endswith(("lora_A", "lora_B")):
                self.decay_mask[off:off + k] = 1
        self.m = np.zeros(n, F32)
        self.v = np.zeros(n, F32)

    def window(self, s, drop, crop):
        ctx = np.zeros((self.tokens, self.lm.cfg.dim), F32)
        if not drop:
            ctx[:s["tokens"]] = s["context"]
        return s["codes"][:, crop:crop + self.frames], ctx

    def _run(self, wins, grads):
        codes = np.stack([w[0] for w in wins]).astype(np.int32)
        ctx = np.stack([w[1] for w in wins]).astype(F32)
        return O.lm_step(self.lm.cfg, self.lm.Wflat, self.ad, self.params, codes, ctx, prefix=self.prefix,
                         grads=grads)

    def evaluate(self):
        probes = self.probes_ or self.samples
        n = len(probes) if self.eval_samples == 0 else min(len(probes), self.eval_samples)
        loss, _ = self._run([self.window(p, self.eval_null, (p["frames"] - self.frames) // 2) for p in probes[:n]],
                            False)
        return float(np.sum(loss.astype(np.float64))) / n

    def train(self, steps):
        g = R.MT19937(self.seed)
        order = list(range(len(self.samples)))
        seen = 0
        out = {"before": self.evaluate(), "steps": []}
        for step in range(1, steps + 1):
            wins = []
            for _ in range(self.accumulation):
                index = seen % len(order)
                if index == 0:
                    R.shuffle(order, g)
                s = self.samples[order[index]]
                drop = R.uniform_real(g) < F32(self.dropout)
                crop = R.uniform_int(g, 0, s["frames"] - self.frames) if self.random_crop else (s["frames"] - self.frames) // 2
                wins.append(self.window(s, drop, crop))
                seen += 1
            loss, grad = self._run(wins, True)
            out["steps"].append(float(np.sum(loss.astype(np.float64))) / self.accumulation)
            lr = O.lib().ora_rate(F32(self.lr), step, self.warmup, int(self.schedule == "inverse"))
            O.lib().ora_adamw(self.params.size, self.params, self.m, self.v, grad.astype(F32), self.decay_mask,
                              self.accumulation, step, lr, self.beta1, self.beta2, self.eps, self.decay, self.clip)
        out["after"] = self.evaluate()
        return out
