"""Builders shared by the GPU parity tests: one set of random weights, adapter values and
inputs, handed both to the CPU oracle (fp32, dequantised) and to libactrain.so (as F32, F16 or
Q8_0 bytes, exactly what a GGUF would carry)."""
from __future__ import annotations

import numpy as np

import actrain as A
import oracle as O


def q8_0_bytes(w: np.ndarray) -> np.ndarray:
    rows = np.ascontiguousarray(w, np.float32).reshape(-1, 32)
    out = np.zeros(rows.shape[0] * 34, np.uint8)
    O.lib().ora_q8_0_quant(np.ascontiguousarray(rows.ravel()), rows.shape[0], out)
    return out


def dequant(blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    O.lib().ora_q8_0_dequant(np.ascontiguousarray(blocks), n // 32, out)
    return out


def _weights(rng, names, shapes, wstd, rope=None):
    W = {}
    for n, (r, c) in zip(names, shapes):
        if n.endswith("rope_freq_factors"):
            w = rope.astype(np.float32)
        elif "norm" in n and n.endswith(".weight"):
            w = (1.0 + 0.1 * rng.standard_normal(c)).astype(np.float32)
        elif "norm" in n or n.endswith(".bias"):
            w = (0.05 * rng.standard_normal(c)).astype(np.float32)
        else:
            w = (wstd * rng.standard_normal((r, c) if r > 1 else c)).astype(np.float32)
        W[n] = w
    return W


def _bind_all(ctx, W, wtype, quantizable):
    """Bind every tensor; returns the fp32 values the oracle must use (dequantised)."""
    used = {}
    for n, w in W.items():
        if quantizable(n) and w.ndim == 2 and wtype == "q8_0" and w.shape[1] % 32 == 0:
            q = q8_0_bytes(w)
            ctx.bind(n, q, A.TYPE_Q8_0)
            used[n] = dequant(q, w.size).reshape(w.shape)
        elif quantizable(n) and w.ndim == 2 and wtype == "f16":
            h = w.astype(np.float16)
            ctx.bind(n, h.view(np.uint16), A.TYPE_F16)
            used[n] = h.astype(np.float32)
        else:
            ctx.bind(n, w, A.TYPE_F32)
            used[n] = w
    return used


class MfCase:
    def __init__(self, dim=128, layers=4, heads=2, ff=256, lat=32, cond=32, tdim=16, T=48, C=8, rank=4,
                 alpha=8.0, dora=False, targets=0x7F, first=0, seed=0, wstd=0.05, wtype="f32", batch=3,
                 device=0, b_std=0.03):
        rng = np.random.default_rng(seed)
        self.cfg = O.DitCfg(dim, layers, heads, dim // heads, ff, lat, cond, tdim, (layers - 1) // 2, 1e-5, 1)
        self.ad = O.Adapter(rank, alpha, int(dora), first, targets)
        names = O.dit_tensor_names(self.cfg)
        shapes = O.dit_tensor_shapes(self.cfg)
        rope = 10000.0 ** (2 * np.arange(32) / 64.0)
        W = _weights(rng, names, shapes, wstd, rope)
        self.ctx = A.Context(A.mf_model(dim, layers, heads, ff, lat, cond, tdim),
                             A.AdapterDesc(A.ADAPTER_DORA_ROWS if dora else A.ADAPTER_LORA, rank, alpha, first,
                                           targets, seed + 17, batch, T, C, 0), device)
        quant = lambda n: ".skip." in n or any(n.endswith(t + ".weight") for t in A.TARGETS) or \
            n.endswith(("in_proj.weight", "out_proj.weight", "cond_proj.weight"))
        used = _bind_all(self.ctx, W, wtype, quant)
        self.ctx.finalize()
        self.Wflat = np.concatenate([used[n].ravel() for n in names]).astype(np.float32)
        v, _, _ = self.ctx.get_params()
        self.init = v.copy()
        self.layout = O.adapter_layout(dim, ff, layers, self.ad)
        if b_std:
            for name, off, shape in self.layout:
                k = int(np.prod(shape))
                if name.endswith("lora_B"):
                    v[off:off + k] = b_std * rng.standard_normal(k)
                elif name.endswith("magnitude"):
                    v[off:off + k] *= 1.0 + 0.05 * rng.standard_normal(k)
        self.params = v.astype(np.float32)
        self.ctx.set_params(self.params)
        self.T, self.C, self.batch = T, C, batch
        self.rng = rng

    def inputs(self, n=None, modes=None):
        n = n or self.batch
        rng = self.rng
        lat, cond = self.cfg.latent_dim, self.cfg.cond_dim
        clean = rng.standard_normal((n, lat, self.T)).astype(np.float32)
        noise = rng.standard_normal((n, lat, self.T)).astype(np.float32)
        hidden = rng.standard_normal((n, self.C, cond)).astype(np.float32)
        t = rng.uniform(0, 1, n).astype(np.float32)
        modes = modes or ["cond", "padded", "null"][:n] + ["cond"] * max(0, n - 3)
        unc = np.array([m == "null" for m in modes], np.int32)
        valid = np.array([self.C // 2 if m == "padded" else -1 for m in modes], np.int32)
        return clean, noise, hidden, t, unc, valid

    def oracle(self, params, inputs):
        return O.dit_step(self.cfg, self.Wflat, self.ad, params, *inputs)


class MgCase:
    def __init__(self, dim=128, layers=2, heads=2, ff=256, n_q=4, card=64, frames=20, C=8, prefix=0, rank=4,
                 alpha=8.0, dora=True, targets=0x7F, first=0, seed=0, wstd=0.05, wtype="f32", batch=2,
                 device=0, b_std=0.03):
        rng = np.random.default_rng(seed)
        self.cfg = O.LmCfg(dim, layers, heads, dim // heads, ff, n_q, card, card, dim // 2 - 1, 10000.0, 1e-5)
        self.ad = O.Adapter(rank, alpha, int(dora), first, targets)
        names = O.lm_tensor_names(self.cfg)
        shapes = O.lm_tensor_shapes(self.cfg)
        W = _weights(rng, names, shapes, wstd)
        for q in range(n_q):  # embeddings are O(1) vectors in the real model
            W[f"lm.emb.{q}.weight"] = (0.5 * rng.standard_normal((card + 1, dim))).astype(np.float32)
        self.ctx = A.Context(A.mg_model(dim, layers, heads, ff, n_q, card),
                             A.AdapterDesc(A.ADAPTER_DORA_ROWS if dora else A.ADAPTER_LORA, rank, alpha, first,
                                           targets, seed + 17, batch, frames, C, prefix), device)
        quant = lambda n: any(n.endswith(t + ".weight") for t in A.TARGETS) or ".head." in n
        used = _bind_all(self.ctx, W, wtype, quant)
        self.ctx.finalize()
        self.Wflat = np.concatenate([used[n].ravel() for n in names]).astype(np.float32)
        v, _, _ = self.ctx.get_params()
        self.init = v.copy()
        self.layout = O.adapter_layout(dim, ff, layers, self.ad, prefix="lm")
        if b_std:
            for name, off, shape in self.layout:
                k = int(np.prod(shape))
                if name.endswith("lora_B"):
                    v[off:off + k] = b_std * rng.standard_normal(k)
                elif name.endswith("magnitude"):
                    v[off:off + k] *= 1.0 + 0.05 * rng.standard_normal(k)
        self.params = v.astype(np.float32)
        self.ctx.set_params(self.params)
        self.frames, self.C, self.prefix, self.batch = frames, C, prefix, batch
        self.rng = rng

    def inputs(self, n=None):
        n = n or self.batch
        codes = self.rng.integers(0, self.cfg.card, (n, self.cfg.n_q, self.frames)).astype(np.int32)
        context = self.rng.standard_normal((n, self.C, self.cfg.dim)).astype(np.float32)
        return codes, context

    def oracle(self, params, inputs):
        return O.lm_step(self.cfg, self.Wflat, self.ad, params, *inputs, prefix=self.prefix)


def grad_metrics(g, ref, layout, kind="l2"):
    """(cosine, global relative L2, worst per-tensor relative error, its tensor name).

    kind "l2":  per-tensor ||g - ref|| / ||ref||            (the parity gate)
    kind "max": per-tensor max|g - ref| / max|ref|           (reported, stricter)"""
    g64, r64 = g.astype(np.float64), ref.astype(np.float64)
    cos = float(np.dot(g64, r64) / (np.linalg.norm(g64) * np.linalg.norm(r64) + 1e-300))
    rel = float(np.linalg.norm(g64 - r64) / (np.linalg.norm(r64) + 1e-300))
    worst, worst_name = 0.0, ""
    for name, off, shape in layout:
        k = int(np.prod(shape))
        r = r64[off:off + k]
        d = g64[off:off + k] - r
        if kind == "l2":
            scale = np.linalg.norm(r)
            e = float(np.linalg.norm(d) / scale) if scale > 0 else 0.0
        else:
            scale = np.abs(r).max()
            e = float(np.abs(d).max() / scale) if scale > 0 else 0.0
        if e > worst:
            worst, worst_name = e, name
    return cos, rel, worst, worst_name
