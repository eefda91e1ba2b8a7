"""Generate the golden fixtures that pin the CPU oracle.

Run from the repository root:  python tests/golden/gen_fixtures.py [--reference DIR]

DIR (or the environment variable AUDIOCRAFT_CPP_REFERENCE) is a checkout of the audiocraft.cpp
tree; without it the delay-pattern goldens already committed are kept.

Three sources, none of them the oracle itself:
  * an fp64 PyTorch restatement of the reference training graph, differentiated by torch
    autograd, with DoRA in the *materialised* form W' = m (W + sBA)/||W + sBA|| that the
    reference's own opt-in oracle uses (tests/mf_train_torch_parity.py:47-56 in the
    audiocraft.cpp tree) -- independent of the hand-derived backward in the C oracle;
  * gguf-py's Q8_0 quantizer (documented there as bit-exact with ggml-quants.c);
  * the delay-pattern arrays of the reference's tests/pattern_test.cpp:93-146, parsed from
    that file when it is present (the reference tree is read-only and only exists in the
    build container, so the parsed arrays are committed as JSON).
"""
from __future__ import annotations

import json
import math
import os
import re
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("AUDIOCRAFT_CPP_REFERENCE", "")
TARGETS = ("self.qkv", "self.out", "cross.q", "cross.kv", "cross.out", "ff.0", "ff.2")

torch.set_default_dtype(torch.float64)

# --------------------------------------------------------------------------------------
# fp64 restatement (autograd)

AS = (0.3275911, 0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def gelu_as(x):
    """src/ac/lora.h:97-110: x * (1/2 + 1/2 sgn(z)(1 - poly(t) e^{-z^2})), z = x/sqrt2."""
    z = x * 0.7071067811865475
    a = torch.abs(z)
    t = 1.0 / (1.0 + AS[0] * a)
    poly = t * (AS[1] + t * (AS[2] + t * (AS[3] + t * (AS[4] + t * AS[5]))))
    erf = torch.sign(z) * (1.0 - poly * torch.exp(-z * z))
    return x * (0.5 + 0.5 * erf)


def layer_norm(x, w, b, eps):
    mu = x.mean(-1, keepdim=True)
    c = x - mu
    return c / torch.sqrt((c * c).mean(-1, keepdim=True) + eps) * w + b


def adapted_weight(W, A, B, m, s):
    direction = W + s * (B @ A)
    if m is None:
        return direction
    nsq = (direction * direction).sum(1, keepdim=True) + W.shape[1] * 1e-12
    return m.reshape(-1, 1) * direction / torch.sqrt(nsq)


def attention(q, k, v, heads, zero_key, key_mask=None, causal=False):
    """q [T, D], k/v [Tk, D] -> [T, D]; heads split on the feature axis."""
    T, D = q.shape
    hd = D // heads
    qh = q.reshape(T, heads, hd).transpose(0, 1)
    kh = k.reshape(-1, heads, hd).transpose(0, 1)
    vh = v.reshape(-1, heads, hd).transpose(0, 1)
    s = qh @ kh.transpose(1, 2) / math.sqrt(hd)
    if key_mask is not None:
        s = s.masked_fill(~key_mask.view(1, 1, -1), -math.inf)
    if causal:
        tri = torch.ones(T, kh.shape[1], dtype=torch.bool).tril()
        s = s.masked_fill(~tri, -math.inf)
    if zero_key:
        s = torch.cat([torch.zeros(heads, T, 1), s], dim=2)
        vh = torch.cat([torch.zeros(heads, 1, hd), vh], dim=1)
    p = torch.softmax(s, dim=-1)
    return (p @ vh).transpose(0, 1).reshape(T, D)


def rope(x, heads, ff):
    """Interleaved pairs rotated by pos / ff[i] (complex form, as audiocraft's RoPE)."""
    T, D = x.shape
    hd = D // heads
    pos = torch.arange(T, dtype=torch.float64).view(T, 1)
    theta = pos / torch.as_tensor(ff, dtype=torch.float64).view(1, -1)       # [T, hd/2]
    xc = torch.view_as_complex(x.reshape(T, heads, hd // 2, 2).contiguous())
    rot = torch.polar(torch.ones_like(theta), theta).view(T, 1, hd // 2)
    return torch.view_as_real(xc * rot).reshape(T, D)


def timestep_features_f32(t, dim, max_period=10000.0):
    """src/ac/transformer.h:144-154 in float32, exactly as the C++ computes it."""
    half = dim // 2
    out = np.zeros(dim, np.float32)
    lmp = np.float32(math.log(np.float32(max_period)))
    for i in range(half):
        freq = np.exp(np.float32(-lmp) * np.float32(i) / np.float32(half), dtype=np.float32)
        arg = np.float32(t) * freq
        out[i] = np.cos(arg, dtype=np.float32)
        out[half + i] = np.sin(arg, dtype=np.float32)
    return out


def skip_plan(idx, layers, n_skip):
    half = layers / 2.0
    cons = n_skip > 0 and idx > half
    prod = n_skip > 0 and idx < half - 1.0
    return cons, prod, (idx % n_skip if cons else 0)


def dit_loss(cfg, Wn, adapters, clean, noise, hidden, t, uncond, valid):
    """One clip of src/mf/train.h:148-188 -> dit_forward (src/mf/dit.h:160-212)."""
    D, H = cfg["dim"], cfg["heads"]
    lat, T = clean.shape
    x_t = (1 - t) * noise + t * clean
    vstar = clean - noise
    rescale = 1.0 / math.sqrt(t * t + (1 - t) * (1 - t))
    x = (x_t.T * rescale) @ Wn["dit.in_proj.weight"].T
    tfeat = torch.from_numpy(timestep_features_f32(np.float32(t), cfg["time_dim"]).astype(np.float64))
    te = torch.nn.functional.silu(Wn["dit.time_embed.0.weight"] @ tfeat)
    te = Wn["dit.time_embed.2.weight"] @ te
    ctx = hidden @ Wn["dit.cond_proj.weight"].T + Wn["dit.cond_proj.bias"]
    C = hidden.shape[0]
    key_mask = torch.zeros(C, dtype=torch.bool)
    if not uncond:
        key_mask[: (C if valid < 0 else valid)] = True
    ff = Wn["dit.rope_freq_factors"]

    def proj(name, inp):
        W = Wn[name]
        if name in adapters:
            A, B, m, s = adapters[name]
            W = adapted_weight(W, A, B, m, s)
        return inp @ W.T

    saved = []
    for idx in range(cfg["layers"]):
        cons, prod, pj = skip_plan(idx, cfg["layers"], cfg["n_skip"])
        if cons:
            x = torch.cat([x, saved.pop()], dim=1) @ Wn[f"dit.skip.{pj}.weight"].T
        p = f"dit.{idx}."
        h = layer_norm(x, Wn[p + "norm1.weight"], Wn[p + "norm1.bias"], cfg["norm_eps"]) + te
        qkv = proj(p + "self.qkv.weight", h)
        q, k, v = qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:]
        o = attention(rope(q, H, ff), rope(k, H, ff), v, H, cfg["add_zero_attn"])
        x = x + proj(p + "self.out.weight", o)
        hc = layer_norm(x, Wn[p + "norm_cross.weight"], Wn[p + "norm_cross.bias"], cfg["norm_eps"]) + te
        cq = proj(p + "cross.q.weight", hc)
        ckv = proj(p + "cross.kv.weight", ctx)
        o2 = attention(cq, ckv[:, :D], ckv[:, D:], H, cfg["add_zero_attn"], key_mask)
        x = x + proj(p + "cross.out.weight", o2)
        f = layer_norm(x, Wn[p + "norm2.weight"], Wn[p + "norm2.bias"], cfg["norm_eps"])
        x = x + proj(p + "ff.2.weight", gelu_as(proj(p + "ff.0.weight", f)))
        if prod:
            saved.append(x)
    x = layer_norm(x, Wn["dit.out_norm.weight"], Wn["dit.out_norm.bias"], cfg["norm_eps"])
    v = (x @ Wn["dit.out_proj.weight"].T).T * math.sqrt(2.0)
    return ((v - vstar) ** 2).mean()


def sin_positions(n, dim, denom, max_period):
    half = dim // 2
    out = np.zeros((n, dim), np.float32)
    for t in range(n):
        for i in range(half):
            ph = t / max_period ** (i / denom)
            out[t, i] = np.float32(math.cos(ph))
            out[t, half + i] = np.float32(math.sin(ph))
    return out


def lm_loss(cfg, Wn, adapters, codes, context, prefix):
    """One sequence of src/mg/train.h:12-49,131,178-227."""
    D, H, nq, card = cfg["dim"], cfg["heads"], cfg["n_q"], cfg["card"]
    frames = codes.shape[1]
    S = 1 + frames + nq - 1
    steps = S - 1
    special = cfg["special_token_id"]
    seq = np.full((nq, S), special, np.int64)
    for q in range(nq):
        for s in range(1, S):
            t = s - 1 - q
            if 0 <= t < frames:
                seq[q, s] = codes[q, t]
    x = sum(Wn[f"lm.emb.{q}.weight"][torch.from_numpy(seq[q, :steps])] for q in range(nq))
    x = x + torch.from_numpy(sin_positions(steps, D, cfg["pos_denominator"],
                                           cfg["max_period"]).astype(np.float64))

    def proj(name, inp):
        W = Wn[name]
        if name in adapters:
            A, B, m, s = adapters[name]
            W = adapted_weight(W, A, B, m, s)
        return inp @ W.T

    for idx in range(cfg["layers"]):
        p = f"lm.{idx}."
        h = layer_norm(x, Wn[p + "norm1.weight"], Wn[p + "norm1.bias"], cfg["norm_eps"])
        qkv = proj(p + "self.qkv.weight", h)
        o = attention(qkv[:, :D], qkv[:, D:2 * D], qkv[:, 2 * D:], H, False, causal=True)
        x = x + proj(p + "self.out.weight", o)
        h = layer_norm(x, Wn[p + "norm_cross.weight"], Wn[p + "norm_cross.bias"], cfg["norm_eps"])
        ckv = proj(p + "cross.kv.weight", context)
        o = attention(proj(p + "cross.q.weight", h), ckv[:, :D], ckv[:, D:], H, False)
        x = x + proj(p + "cross.out.weight", o)
        h = layer_norm(x, Wn[p + "norm2.weight"], Wn[p + "norm2.bias"], cfg["norm_eps"])
        x = x + proj(p + "ff.2.weight", gelu_as(proj(p + "ff.0.weight", h)))
    x = layer_norm(x, Wn["lm.out_norm.weight"], Wn["lm.out_norm.bias"], cfg["norm_eps"])
    rows, targets = [], []
    for q in range(nq):
        logits = x @ Wn[f"lm.head.{q}.weight"].T
        for s in range(steps):
            t = s - q  # timestep at step s+1 for codebook q
            if prefix <= t < frames:
                rows.append(logits[s])
                targets.append(int(codes[q, t]))
    logits = torch.stack(rows)
    return torch.nn.functional.cross_entropy(logits, torch.tensor(targets), reduction="mean")


# --------------------------------------------------------------------------------------
# fixture assembly

def dit_names(cfg):
    names = ["dit.in_proj.weight", "dit.out_proj.weight", "dit.time_embed.0.weight",
             "dit.time_embed.2.weight", "dit.cond_proj.weight", "dit.cond_proj.bias",
             "dit.rope_freq_factors", "dit.out_norm.weight", "dit.out_norm.bias"]
    names += [f"dit.skip.{i}.weight" for i in range(cfg["n_skip"])]
    for l in range(cfg["layers"]):
        for n in ("norm1", "norm_cross", "norm2"):
            names += [f"dit.{l}.{n}.weight", f"dit.{l}.{n}.bias"]
        names += [f"dit.{l}.{t}.weight" for t in TARGETS]
    return names


def dit_shape(cfg, name):
    D, F = cfg["dim"], cfg["ff_dim"]
    table = {"dit.in_proj.weight": (D, cfg["latent_dim"]), "dit.out_proj.weight": (cfg["latent_dim"], D),
             "dit.time_embed.0.weight": (D, cfg["time_dim"]), "dit.time_embed.2.weight": (D, D),
             "dit.cond_proj.weight": (D, cfg["cond_dim"]), "dit.cond_proj.bias": (D,),
             "dit.rope_freq_factors": (cfg["head_dim"] // 2,)}
    if name in table:
        return table[name]
    if ".skip." in name:
        return (D, 2 * D)
    if "norm" in name:
        return (D,)
    return proj_shape(name, D, F)


def proj_shape(name, D, F):
    t = name.split(".", 2)[2].rsplit(".", 1)[0]
    return {"self.qkv": (3 * D, D), "self.out": (D, D), "cross.q": (D, D),
            "cross.kv": (2 * D, D), "cross.out": (D, D), "ff.0": (F, D), "ff.2": (D, F)}[t]


def lm_names(cfg):
    names = [f"lm.emb.{q}.weight" for q in range(cfg["n_q"])]
    names += [f"lm.head.{q}.weight" for q in range(cfg["n_q"])]
    names += ["lm.out_norm.weight", "lm.out_norm.bias"]
    for l in range(cfg["layers"]):
        for n in ("norm1", "norm_cross", "norm2"):
            names += [f"lm.{l}.{n}.weight", f"lm.{l}.{n}.bias"]
        names += [f"lm.{l}.{t}.weight" for t in TARGETS]
    return names


def lm_shape(cfg, name):
    D, F = cfg["dim"], cfg["ff_dim"]
    if ".emb." in name:
        return (cfg["card"] + 1, D)
    if ".head." in name:
        return (cfg["card"], D)
    if "norm" in name:
        return (D,)
    return proj_shape(name, D, F)


def make_weights(rng, names, shape_fn, std, rope_ff=None):
    out = {}
    for n in names:
        shp = shape_fn(n)
        if n.endswith("rope_freq_factors"):
            w = rope_ff.astype(np.float32)
        elif "norm" in n and n.endswith(".weight"):
            w = (1.0 + 0.1 * rng.standard_normal(shp)).astype(np.float32)
        elif "norm" in n or n.endswith(".bias"):
            w = (0.05 * rng.standard_normal(shp)).astype(np.float32)
        else:
            w = (std * rng.standard_normal(shp)).astype(np.float32)
        out[n] = w
    return out


def adapter_entries(prefix, layers, first, targets, rank, D, F, dora):
    out = []
    for l in range(first, layers):
        for t in range(7):
            if not (targets >> t) & 1:
                continue
            stem = f"{prefix}.{l}.{TARGETS[t]}.weight"
            o, i = proj_shape(stem, D, F)
            out.append((stem, (rank, i), (o, rank), (o,) if dora else None))
    return out


def make_params(rng, entries, Wnp, zero_b, dora):
    vals = []
    for stem, sa, sb, sm in entries:
        A = (0.02 * rng.standard_normal(sa)).astype(np.float32)
        B = np.zeros(sb, np.float32) if zero_b else (0.03 * rng.standard_normal(sb)).astype(np.float32)
        vals += [A.ravel(), B.ravel()]
        if dora:
            W = Wnp[stem].astype(np.float64)
            m = np.sqrt((W * W).sum(1) + W.shape[1] * 1e-12)
            if not zero_b:
                m = m * (1.0 + 0.05 * rng.standard_normal(m.shape))
            vals.append(m.astype(np.float32))
    return np.concatenate(vals)


def split_params(flat, entries, s, requires_grad=True):
    adapters, leaves, off = {}, [], 0
    for stem, sa, sb, sm in entries:
        parts = []
        for shp in (sa, sb) + ((sm,) if sm else ()):
            n = int(np.prod(shp))
            t = torch.from_numpy(flat[off:off + n].astype(np.float64)).reshape(shp)
            t.requires_grad_(requires_grad)
            parts.append(t)
            leaves.append(t)
            off += n
        adapters[stem] = (parts[0], parts[1], parts[2] if sm else None, s)
    return adapters, leaves


def dit_case(name, cfg, T, C, rank, alpha, dora, zero_b, first, targets, clips, seed):
    rng = np.random.default_rng(seed)
    names = dit_names(cfg)
    hd = cfg["head_dim"]
    ff = np.array([10000.0 ** (2 * i / hd) for i in range(hd // 2)], np.float32)
    Wnp = make_weights(rng, names, lambda n: dit_shape(cfg, n), 0.15, ff)
    entries = adapter_entries("dit", cfg["layers"], first, targets, rank, cfg["dim"], cfg["ff_dim"], dora)
    params = make_params(rng, entries, Wnp, zero_b, dora)
    n = len(clips)
    lat = cfg["latent_dim"]
    clean = rng.standard_normal((n, lat, T)).astype(np.float32)
    noise = rng.standard_normal((n, lat, T)).astype(np.float32)
    hidden = rng.standard_normal((n, C, cfg["cond_dim"])).astype(np.float32)
    tv = np.array([c[0] for c in clips], np.float32)
    uncond = np.array([c[1] for c in clips], np.int32)
    valid = np.array([c[2] for c in clips], np.int32)
    Wn = {k: torch.from_numpy(v.astype(np.float64)) for k, v in Wnp.items()}
    adapters, leaves = split_params(params, entries, alpha / rank)
    losses = []
    total = 0
    for b in range(n):
        l = dit_loss(cfg, Wn, adapters, torch.from_numpy(clean[b].astype(np.float64)),
                     torch.from_numpy(noise[b].astype(np.float64)),
                     torch.from_numpy(hidden[b].astype(np.float64)), float(tv[b]), bool(uncond[b]),
                     int(valid[b]))
        losses.append(l.item())
        total = total + l
    total.backward()
    grads = np.concatenate([p.grad.numpy().ravel() for p in leaves])
    W = np.concatenate([Wnp[k].ravel() for k in names])
    np.savez_compressed(os.path.join(HERE, f"dit_{name}.npz"), kind="dit",
                        cfg=json.dumps(cfg), T=T, C=C, rank=rank, alpha=alpha, dora=int(dora),
                        first_layer=first, targets=targets, W=W, params=params, clean=clean,
                        noise=noise, hidden=hidden, t=tv, uncond=uncond, valid=valid,
                        loss=np.array(losses), grads=grads)
    print(f"dit_{name}: loss {losses} |g| {np.linalg.norm(grads):.4g}")


def lm_case(name, cfg, frames, C, prefix, rank, alpha, dora, zero_b, first, targets, nseq, seed):
    rng = np.random.default_rng(seed)
    names = lm_names(cfg)
    Wnp = make_weights(rng, names, lambda n: lm_shape(cfg, n), 0.15)
    entries = adapter_entries("lm", cfg["layers"], first, targets, rank, cfg["dim"], cfg["ff_dim"], dora)
    params = make_params(rng, entries, Wnp, zero_b, dora)
    codes = rng.integers(0, cfg["card"], (nseq, cfg["n_q"], frames)).astype(np.int32)
    context = rng.standard_normal((nseq, C, cfg["dim"])).astype(np.float32)
    Wn = {k: torch.from_numpy(v.astype(np.float64)) for k, v in Wnp.items()}
    adapters, leaves = split_params(params, entries, alpha / rank)
    losses, total = [], 0
    for b in range(nseq):
        l = lm_loss(cfg, Wn, adapters, codes[b], torch.from_numpy(context[b].astype(np.float64)), prefix)
        losses.append(l.item())
        total = total + l
    total.backward()
    grads = np.concatenate([p.grad.numpy().ravel() for p in leaves])
    W = np.concatenate([Wnp[k].ravel() for k in names])
    np.savez_compressed(os.path.join(HERE, f"lm_{name}.npz"), kind="lm", cfg=json.dumps(cfg),
                        frames=frames, C=C, prefix=prefix, rank=rank, alpha=alpha, dora=int(dora),
                        first_layer=first, targets=targets, W=W, params=params, codes=codes,
                        context=context, loss=np.array(losses), grads=grads)
    print(f"lm_{name}: loss {losses} |g| {np.linalg.norm(grads):.4g}")


def q8_fixture():
    from gguf.quants import Q8_0
    rng = np.random.default_rng(7)
    blocks = [rng.standard_normal(32) * 0.02, rng.standard_normal(32) * 3.0, np.zeros(32),
              np.linspace(-1, 1, 32), np.full(32, 1e-6), rng.standard_normal(32) * 1e-4,
              np.array([127.0 * (k - 16) / 16 + 0.5 for k in range(32)]),  # exact .5 ties
              rng.standard_normal(32) * 60000.0 / 127]
    for _ in range(56):
        blocks.append(rng.standard_normal(32) * 10 ** rng.uniform(-4, 1))
    x = np.stack(blocks).astype(np.float32)
    q = Q8_0.quantize_blocks(x)
    deq = Q8_0.dequantize_blocks(q).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q8_0.npz"), x=x, q=q.astype(np.uint8), deq=deq)
    print("q8_0: blocks", x.shape[0])


def pattern_fixture():
    path = os.path.join(REF, "tests", "pattern_test.cpp") if REF else ""
    out = os.path.join(HERE, "pattern_goldens.json")
    if not path or not os.path.exists(path):
        print("pattern goldens: reference tree absent, keeping committed JSON")
        return
    text = open(path).read()
    cases = {}
    for m in re.finditer(r"constexpr int (\w+)_NQ = (\d+), \w+_T = (\d+), \w+_S = (\d+), \w+_SPECIAL = (\d+);", text):
        tag = m.group(1)
        case = {"n_q": int(m.group(2)), "T": int(m.group(3)), "S": int(m.group(4)),
                "special": int(m.group(5))}
        for arr in ("codes", "sequence", "mask", "reverted", "first_step"):
            mm = re.search(rf"{tag}_{arr}\[\] = \{{(.*?)\}};", text, re.S)
            case[arr] = [int(v) for v in mm.group(1).replace("\n", " ").split(",") if v.strip()]
        cases[tag] = case
    src = {"source": "audiocraft.cpp tests/pattern_test.cpp:93-146 (DelayedPatternProvider goldens)",
           "cases": cases}
    json.dump(src, open(out, "w"), indent=1)
    print("pattern goldens:", list(cases))


def main():
    global REF
    if "--reference" in sys.argv:
        REF = sys.argv[sys.argv.index("--reference") + 1]
    tiny = dict(dim=8, layers=4, heads=2, head_dim=4, ff_dim=16, latent_dim=4, cond_dim=6,
                time_dim=8, n_skip=1, norm_eps=1e-5, add_zero_attn=True)
    small = dict(dim=16, layers=6, heads=2, head_dim=8, ff_dim=32, latent_dim=4, cond_dim=6,
                 time_dim=8, n_skip=2, norm_eps=1e-5, add_zero_attn=True)
    clips3 = [(0.43, 0, -1), (0.81, 0, 1), (0.12, 1, -1)]   # conditional, padded, null
    dit_case("tiny_lora_zeroB", tiny, 3, 2, 2, 2.0, False, True, 0, 0x1F, [(0.43, 0, -1)], 1)
    dit_case("tiny_lora", tiny, 3, 2, 2, 2.0, False, False, 0, 0x7F, clips3, 2)
    dit_case("tiny_dora", tiny, 3, 2, 2, 2.0, True, False, 0, 0x7F, clips3, 3)
    dit_case("small_lora", small, 7, 3, 2, 2.0, False, False, 0, 0x7F, clips3, 4)
    dit_case("small_dora", small, 7, 3, 2, 2.0, True, False, 0, 0x7F, clips3, 5)
    dit_case("small_dora_zeroB_l2", small, 7, 3, 2, 2.0, True, True, 2, 0x1F, clips3, 6)
    dit_case("small_lora_r4_a8", small, 9, 3, 4, 8.0, False, False, 3, 0x63, clips3[:2], 7)
    lmc = dict(dim=16, layers=2, heads=2, head_dim=8, ff_dim=32, n_q=4, card=11,
               special_token_id=11, pos_denominator=7, max_period=10000.0, norm_eps=1e-5)
    lm_case("tiny_lora", lmc, 7, 3, 0, 2, 2.0, False, False, 0, 0x7F, 2, 11)
    lm_case("tiny_dora", lmc, 7, 3, 0, 2, 2.0, True, False, 0, 0x7F, 2, 12)
    lm_case("tiny_dora_prefix", lmc, 7, 3, 2, 2, 2.0, True, False, 1, 0x1F, 1, 13)
    q8_fixture()
    pattern_fixture()


if __name__ == "__main__":
    sys.exit(main())
