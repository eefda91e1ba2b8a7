"""ctypes view of the CPU restatement in actrain_oracle.c.

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by the
CPU-baseline leg of bench.py, always as the checker.  The product never imports this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

TARGETS = ("self.qkv", "self.out", "cross.q", "cross.kv", "cross.out", "ff.0", "ff.2")
REFERENCE_TARGETS = 0x1F          # src/mf/train.h:69-70 without --train-ffn
REFERENCE_TARGETS_FFN = 0x7F      # with --train-ffn


class DitCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "layers", "heads", "head_dim", "ff_dim",
                                        "latent_dim", "cond_dim", "time_dim", "n_skip")] + \
               [("norm_eps", C.c_float), ("add_zero_attn", C.c_int)]


class LmCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("dim", "layers", "heads", "head_dim", "ff_dim", "n_q",
                                        "card", "special_token_id", "pos_denominator")] + \
               [("max_period", C.c_float), ("norm_eps", C.c_float)]


class Adapter(C.Structure):
    _fields_ = [("rank", C.c_int), ("alpha", C.c_float), ("dora", C.c_int),
                ("first_layer", C.c_int), ("targets", C.c_uint)]


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        L.ora_q8_0_dequant.argtypes = [u8p, C.c_int64, f32p]
        L.ora_q8_0_quant.argtypes = [f32p, C.c_int64, u8p]
        L.ora_half_to_float.argtypes = [C.c_uint16]
        L.ora_half_to_float.restype = C.c_float
        L.ora_float_to_half.argtypes = [C.c_float]
        L.ora_float_to_half.restype = C.c_uint16
        L.ora_skip_plan.argtypes = [C.c_int, C.c_int, C.c_int] + [C.POINTER(C.c_int)] * 3
        L.ora_timestep_features.argtypes = [C.c_float, C.c_int, C.c_float, f32p]
        L.ora_dit_input_rescale.argtypes = [C.c_float]
        L.ora_dit_input_rescale.restype = C.c_float
        L.ora_sin_positions.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, f32p]
        L.ora_pattern_build.argtypes = [C.c_int, C.c_int, i32p, C.c_int32, i32p]
        L.ora_pattern_revert.argtypes = [C.c_int, C.c_int, i32p, C.c_int32, i32p]
        L.ora_pattern_mask.argtypes = [C.c_int, C.c_int, u8p]
        L.ora_gelu.argtypes = [C.c_float]
        L.ora_gelu.restype = C.c_float
        L.ora_gelu_grad.argtypes = [C.c_float]
        L.ora_gelu_grad.restype = C.c_float
        L.ora_row_norm_sq.argtypes = [f32p, C.c_int, C.c_int, f32p]
        L.ora_adapter_numel.argtypes = [C.c_int, C.c_int, C.c_int, C.POINTER(Adapter)]
        L.ora_adapter_numel.restype = C.c_int64
        L.ora_dit_tensor_count.argtypes = [C.POINTER(DitCfg)]
        L.ora_dit_tensor_shape.argtypes = [C.POINTER(DitCfg), C.c_int, C.POINTER(C.c_int),
                                           C.POINTER(C.c_int)]
        L.ora_dit_tensor_shape.restype = C.c_int64
        L.ora_lm_tensor_count.argtypes = [C.POINTER(LmCfg)]
        L.ora_lm_tensor_shape.argtypes = [C.POINTER(LmCfg), C.c_int, C.POINTER(C.c_int),
                                          C.POINTER(C.c_int)]
        L.ora_lm_tensor_shape.restype = C.c_int64
        L.ora_dit_step.argtypes = [C.POINTER(DitCfg), f32p, C.POINTER(Adapter), f32p, C.c_int,
                                   C.c_int, C.c_int, f32p, f32p, f32p, f32p, i32p, i32p, f32p,
                                   C.c_void_p]
        L.ora_lm_step.argtypes = [C.POINTER(LmCfg), f32p, C.POINTER(Adapter), f32p, C.c_int,
                                  C.c_int, C.c_int, C.c_int, i32p, f32p, f32p, C.c_void_p]
        L.ora_rate.argtypes = [C.c_float, C.c_int, C.c_int, C.c_int]
        L.ora_rate.restype = C.c_float
        L.ora_adamw.argtypes = [C.c_int64, f32p, f32p, f32p, f32p, u8p, C.c_int, C.c_int,
                                C.c_float, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float]
        L.ora_adamw.restype = C.c_int64
        L.ora_target_suffix.argtypes = [C.c_int]
        L.ora_target_suffix.restype = C.c_char_p
        _lib = L
    return _lib


# ---------------------------------------------------------------------------------------
# convenience wrappers

def dit_tensor_names(cfg: DitCfg) -> list[str]:
    names = ["dit.in_proj.weight", "dit.out_proj.weight", "dit.time_embed.0.weight",
             "dit.time_embed.2.weight", "dit.cond_proj.weight", "dit.cond_proj.bias",
             "dit.rope_freq_factors", "dit.out_norm.weight", "dit.out_norm.bias"]
    names += [f"dit.skip.{i}.weight" for i in range(cfg.n_skip)]
    for l in range(cfg.layers):
        p = f"dit.{l}."
        for n in ("norm1", "norm_cross", "norm2"):
            names += [p + n + ".weight", p + n + ".bias"]
        names += [p + t + ".weight" for t in TARGETS]
    return names


def lm_tensor_names(cfg: LmCfg) -> list[str]:
    names = [f"lm.emb.{q}.weight" for q in range(cfg.n_q)]
    names += [f"lm.head.{q}.weight" for q in range(cfg.n_q)]
    names += ["lm.out_norm.weight", "lm.out_norm.bias"]
    for l in range(cfg.layers):
        p = f"lm.{l}."
        for n in ("norm1", "norm_cross", "norm2"):
            names += [p + n + ".weight", p + n + ".bias"]
        names += [p + t + ".weight" for t in TARGETS]
    return names


def dit_tensor_shapes(cfg: DitCfg) -> list[tuple[int, int]]:
    L = lib()
    out = []
    for i in range(L.ora_dit_tensor_count(C.byref(cfg))):
        r, k = C.c_int(), C.c_int()
        L.ora_dit_tensor_shape(C.byref(cfg), i, C.byref(r), C.byref(k))
        out.append((r.value, k.value))
    return out


def lm_tensor_shapes(cfg: LmCfg) -> list[tuple[int, int]]:
    L = lib()
    out = []
    for i in range(L.ora_lm_tensor_count(C.byref(cfg))):
        r, k = C.c_int(), C.c_int()
        L.ora_lm_tensor_shape(C.byref(cfg), i, C.byref(r), C.byref(k))
        out.append((r.value, k.value))
    return out


def adapter_layout(D: int, F: int, layers: int, ad: Adapter, prefix: str = "dit"):
    """[(name, offset, shape)] in the reference parameter order (src/mf/train.h:68-104)."""
    ins = {0: D, 1: D, 2: D, 3: D, 4: D, 5: D, 6: F}
    outs = {0: 3 * D, 1: D, 2: D, 3: 2 * D, 4: D, 5: F, 6: D}
    off, out = 0, []
    for l in range(ad.first_layer, layers):
        for t in range(7):
            if not (ad.targets >> t) & 1:
                continue
            stem = f"{prefix}.{l}.{TARGETS[t]}.weight"
            for kind, shape in (("lora_A", (ad.rank, ins[t])), ("lora_B", (outs[t], ad.rank))) + \
                    ((("magnitude", (outs[t],)),) if ad.dora else ()):
                n = int(np.prod(shape))
                out.append((f"{stem}.{kind}", off, shape))
                off += n
    return out


def dit_step(cfg, W, ad, params, clean, noise, hidden, t, uncond, valid, grads=True):
    n, lat, T = clean.shape
    Cn = hidden.shape[1]
    loss = np.zeros(n, np.float32)
    g = np.zeros_like(params) if grads else None
    rc = lib().ora_dit_step(C.byref(cfg), W, C.byref(ad), params, n, T, Cn,
                            np.ascontiguousarray(clean, np.float32),
                            np.ascontiguousarray(noise, np.float32),
                            np.ascontiguousarray(hidden, np.float32),
                            np.ascontiguousarray(t, np.float32),
                            np.ascontiguousarray(uncond, np.int32),
                            np.ascontiguousarray(valid, np.int32), loss,
                            g.ctypes.data if grads else None)
    if rc != 0:
        raise RuntimeError(f"ora_dit_step failed: {rc}")
    return loss, g


def lm_step(cfg, W, ad, params, codes, context, prefix=0, grads=True):
    n, nq, frames = codes.shape
    Cn = context.shape[1]
    loss = np.zeros(n, np.float32)
    g = np.zeros_like(params) if grads else None
    rc = lib().ora_lm_step(C.byref(cfg), W, C.byref(ad), params, n, frames, prefix, Cn,
                           np.ascontiguousarray(codes, np.int32),
                           np.ascontiguousarray(context, np.float32), loss,
                           g.ctypes.data if grads else None)
    if rc != 0:
        raise RuntimeError(f"ora_lm_step failed: {rc}")
    return loss, g
