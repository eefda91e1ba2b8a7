"""Benchmark of the adapter training step (BASELINE.json metric: DiT LoRA train steps/s on
8 x 30 s clips).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload mf|mf-cfg1|mg]

N > 1 is launched by torchrun (one process per GPU).  Per-GPU work is fixed (8 clips of 750
frames per rank, weak scaling) and `value` is the whole-job rate in units of 8-clip steps:
N * K / (max over ranks of the device time of K steps).  Synthetic inputs and N(0, 0.02)
weights quantised to Q8_0 stand in for the reference's datasets and checkpoints.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "audiocraft.cpp_b200"))

# BASELINE cfg 2: DiT d1024 x24, 16 heads, FFN 4096, 8 x 750 frames, 32 T5 tokens, rank 16
# LoRA (alpha 32) on self.qkv, self.out, ff.0, ff.2.
MF = dict(dim=1024, layers=24, heads=16, ff=4096, lat=128, cond=768, tdim=256, T=750, C=32, batch=8,
          rank=16, alpha=32.0, targets=0x63)
# BASELINE cfg 1: the same model with an F16 base, one 250-frame clip and 16 tokens per step.
MF1 = dict(MF, T=250, C=16, batch=1, weights="f16")
# BASELINE cfg 4 (per GPU): MusicGen-medium d1536 x48, 24 heads, FFN 6144, 4 codebooks of 2048,
# 1500 frames, 32 tokens, DoRA-rows rank 16 on all seven projections, 4 sequences per GPU.
MG = dict(dim=1536, layers=48, heads=24, ff=6144, n_q=4, card=2048, frames=1500, C=32, batch=4,
          rank=16, alpha=32.0, targets=0x7F)


def q8_0(w: np.ndarray) -> np.ndarray:
    """ggml quantize_row_q8_0 on rows of 32 (d = amax/127 in fp32, q = round half away)."""
    x = w.reshape(-1, 32).astype(np.float32)
    d = np.abs(x).max(axis=1, keepdims=True) / np.float32(127)
    with np.errstate(divide="ignore"):
        inv = np.where(d == 0, np.float32(0), np.float32(1) / d).astype(np.float32)
    a = np.abs(x * inv)
    fl = np.floor(a)
    q = (np.sign(x) * (fl + np.floor(2 * (a - fl)))).astype(np.int8)
    out = np.empty((x.shape[0], 34), np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.ravel()


def dit_tensors(c):
    D, F = c["dim"], c["ff"]
    t = [("dit.in_proj.weight", (D, c["lat"])), ("dit.out_proj.weight", (c["lat"], D)),
         ("dit.time_embed.0.weight", (D, c["tdim"])), ("dit.time_embed.2.weight", (D, D)),
         ("dit.cond_proj.weight", (D, c["cond"])), ("dit.cond_proj.bias", (D,)),
         ("dit.rope_freq_factors", (32,)), ("dit.out_norm.weight", (D,)), ("dit.out_norm.bias", (D,))]
    t += [(f"dit.skip.{i}.weight", (D, 2 * D)) for i in range((c["layers"] - 1) // 2)]
    for l in range(c["layers"]):
        for n in ("norm1", "norm_cross", "norm2"):
            t += [(f"dit.{l}.{n}.weight", (D,)), (f"dit.{l}.{n}.bias", (D,))]
        t += [(f"dit.{l}.self.qkv.weight", (3 * D, D)), (f"dit.{l}.self.out.weight", (D, D)),
              (f"dit.{l}.cross.q.weight", (D, D)), (f"dit.{l}.cross.kv.weight", (2 * D, D)),
              (f"dit.{l}.cross.out.weight", (D, D)), (f"dit.{l}.ff.0.weight", (F, D)),
              (f"dit.{l}.ff.2.weight", (D, F))]
    return t


def lm_tensors(c):
    D, F = c["dim"], c["ff"]
    t = [(f"lm.emb.{q}.weight", (c["card"] + 1, D)) for q in range(c["n_q"])]
    t += [(f"lm.head.{q}.weight", (c["card"], D)) for q in range(c["n_q"])]
    t += [("lm.out_norm.weight", (D,)), ("lm.out_norm.bias", (D,))]
    for l in range(c["layers"]):
        for n in ("norm1", "norm_cross", "norm2"):
            t += [(f"lm.{l}.{n}.weight", (D,)), (f"lm.{l}.{n}.bias", (D,))]
        t += [(f"lm.{l}.self.qkv.weight", (3 * D, D)), (f"lm.{l}.self.out.weight", (D, D)),
              (f"lm.{l}.cross.q.weight", (D, D)), (f"lm.{l}.cross.kv.weight", (2 * D, D)),
              (f"lm.{l}.cross.out.weight", (D, D)), (f"lm.{l}.ff.0.weight", (F, D)),
              (f"lm.{l}.ff.2.weight", (D, F))]
    return t


def synth_weight(rng, name, shape):
    if name.endswith("rope_freq_factors"):
        return (10000.0 ** (2 * np.arange(32) / 64.0)).astype(np.float32), "f32"
    if "norm" in name:
        return (np.ones(shape) if name.endswith("weight") else np.zeros(shape)).astype(np.float32), "f32"
    if name.endswith(".bias"):
        return np.zeros(shape, np.float32), "f32"
    if ".emb." in name:
        return rng.standard_normal(shape, dtype=np.float32), "f32"
    return (0.02 * rng.standard_normal(shape, dtype=np.float32)), "q8_0"


# ------------------------------------------------------------------------------------------
# clocks

class Clocks:
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------
# CPU baseline: the C restatement (oracle/), the reference binary being unbuildable here

_CPU_MODEL = {}


def cpu_sample(c):
    """One bounded sample of the step on the host cores: forward + backward of ONE clip through
    the full-depth model (all layers, full width and length) in the oracle, the C restatement of
    the reference step.  Clips are independent, so the 8-clip step costs exactly clips x this
    (the optimizer update, 28 bytes per adapter parameter, is noise next to it).  Returns
    (seconds, clips per step, description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if "frames" in c:
        return cpu_sample_lm(c, O)
    L = c["layers"]
    key = (c["dim"], L, c["ff"], c["T"])
    if key not in _CPU_MODEL:  # weights and adapters once per process (1.6 GB of fp32 at cfg 2)
        cfg = O.DitCfg(c["dim"], L, c["heads"], 64, c["ff"], c["lat"], c["cond"], c["tdim"], (L - 1) // 2, 1e-5, 1)
        rng = np.random.default_rng(0)
        shapes = O.dit_tensor_shapes(cfg)
        W = (0.02 * rng.standard_normal(sum(r * k for r, k in shapes), dtype=np.float32))
        ad = O.Adapter(c["rank"], c["alpha"], 0, 0, c["targets"])
        p = (0.02 * rng.standard_normal(O.lib().ora_adapter_numel(c["dim"], c["ff"], L, ad))).astype(np.float32)
        T = c["T"]
        args = (rng.standard_normal((1, c["lat"], T)).astype(np.float32),
                rng.standard_normal((1, c["lat"], T)).astype(np.float32),
                rng.standard_normal((1, c["C"], c["cond"])).astype(np.float32), np.array([0.5], np.float32),
                np.zeros(1, np.int32), np.full(1, -1, np.int32))
        _CPU_MODEL[key] = (cfg, W, ad, p, args)
    cfg, W, ad, p, args = _CPU_MODEL[key]
    t0 = time.perf_counter()
    O.dit_step(cfg, W, ad, p, *args)
    dt = time.perf_counter() - t0
    desc = (f"oracle C restatement (reference binary unbuildable: ggml absent), 1 clip x all {L} layers at "
            f"d{c['dim']} T{c['T']}, fwd+bwd; a step is {c['batch']} such clips")
    return dt, c["batch"], desc


MG_SAMPLE_LAYERS = 12


def cpu_sample_lm(c, O):
    """The MusicGen step's bounded sample: one sequence (all frames, full width) through
    MG_SAMPLE_LAYERS of the model's identical transformer layers, forward + backward, with the
    embeddings, output norm and the four codebook heads.  The layers cost the same, so the full
    step is clips x layers / MG_SAMPLE_LAYERS x this (which counts the embeddings and heads a few
    times over: an overestimate of the CPU step of about 2%)."""
    Ls = min(MG_SAMPLE_LAYERS, c["layers"])
    key = ("lm", c["dim"], Ls, c["ff"], c["frames"])
    if key not in _CPU_MODEL:
        D = c["dim"]
        cfg = O.LmCfg(D, Ls, c["heads"], D // c["heads"], c["ff"], c["n_q"], c["card"], c["card"], D // 2 - 1,
                      10000.0, 1e-5)
        rng = np.random.default_rng(0)
        W = 0.02 * rng.standard_normal(sum(r * k for r, k in O.lm_tensor_shapes(cfg)), dtype=np.float32)
        ad = O.Adapter(c["rank"], c["alpha"], 1, 0, c["targets"])
        p = (0.02 * rng.standard_normal(O.lib().ora_adapter_numel(D, c["ff"], Ls, ad))).astype(np.float32)
        args = (rng.integers(0, c["card"], (1, c["n_q"], c["frames"])).astype(np.int32),
                rng.standard_normal((1, c["C"], D)).astype(np.float32))
        _CPU_MODEL[key] = (cfg, W, ad, p, args)
    cfg, W, ad, p, args = _CPU_MODEL[key]
    t0 = time.perf_counter()
    O.lm_step(cfg, W, ad, p, *args)
    dt = time.perf_counter() - t0
    scale = c["batch"] * c["layers"] / Ls
    desc = (f"oracle C restatement (reference binary unbuildable: ggml absent), 1 sequence x {Ls} of "
            f"{c['layers']} layers at d{c['dim']} {c['frames']} frames, DoRA rows, fwd+bwd; a step is "
            f"{c['batch']} sequences x {c['layers']} layers, value scaled by sample_scale = {scale:g}")
    return dt, scale, desc


def line_header(args, c, n, world):
    """metric, unit and config shared by both arms (the driver compares their values)."""
    mf = args.workload.startswith("mf")
    if args.workload == "mf-cfg1":
        unit = "steps/s (1x10s-clip steps, summed over ranks)"
        metric = "DiT LoRA train steps/s (1x10s clip, F16 base)"
        work = ("mf-cfg1: DiT d1024 L24 H16 F4096 F16 base, 1x250 frames/rank, 16 tokens, "
                "LoRA r16 a32 on qkv/out/ff.0/ff.2, AdamW")
    elif mf:
        unit = "steps/s (8x30s-clip steps, summed over ranks)"
        metric = "DiT LoRA train steps/s (8x30s clips)"
        work = ("mf-cfg2: DiT d1024 L24 H16 F4096 Q8_0 base, 8x750 frames/rank, 32 tokens, "
                "LoRA r16 a32 on qkv/out/ff.0/ff.2 (6,291,456 params), AdamW")
    else:
        unit = "steps/s (4-seq steps, summed over ranks)"
        metric = "MusicGen DoRA train steps/s (4x30s seqs per GPU)"
        work = "mg-cfg4: LM d1536 L48 H24 F6144 Q8_0 base, 4x1500 frames/rank, DoRA-rows r16 on 7 projections"
    config = {"workload": work,
              "global_batch": n * world, "seq_len": c.get("T", c.get("frames")),
              "layers": c["layers"], "clips_per_rank": n,
              "parallelism": f"dp{world}",
              "l2": "no flush: the per-step working set (activations and frozen weights, GBs) exceeds the 126 MB L2"}
    return metric, unit, config


def run_reference(args, c):
    """The reference arm: the reference's step on the host cores, here the oracle restatement
    (the reference binary needs the absent ggml fork).  Each step is one bounded sample, one
    clip of the full-depth model; `ms_per_step` is that sample's time, and `value` scales it by
    `sample_scale` (clips per step) to the metric's 8-clip steps."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count()
    for _ in range(args.warmup):
        cpu_sample(c)
    times = []
    for _ in range(args.steps):
        dt, scale, desc = cpu_sample(c)
        times.append(dt)
    sample_s = float(np.mean(times))
    value = 1.0 / (sample_s * scale)
    metric, unit, config = line_header(args, c, c["batch"], max(args.gpus, 1))
    config = dict(config, sample=desc)
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sample_s * 1e3, "sample_scale": scale,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": config,
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": desc},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------------------------

def run_sweep(kind, reps):
    """Kernel-level sweep (BASELINE cfg 5): one JSON line per shape, device time per call."""
    import actrain as A
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak = peaks.get("bf16_tflops", 1590.0)
    rng = np.random.default_rng(0)
    bits = lambda shape: (rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16) ^
                          (rng.integers(0, 2, size=shape, dtype=np.uint16) << 15))
    if kind == "gemm":
        one = os.environ.get("SWEEP_SHAPE")  # "M,N,K": a single shape (profiling captures)
        for M in ((int(one.split(",")[0]),) if one else (6000,) if os.environ.get("SWEEP_QUICK") else (6000, 2048, 32768)):
            for (N, K) in (((int(one.split(",")[1]), int(one.split(",")[2])),) if one else
                           ((1024, 1024), (3072, 1024), (4096, 1024), (1024, 4096), (1536, 1536), (6144, 1536),
                            (1536, 6144))):
                for b_mn in ((False,) if one else (False, True)):
                    for path in ((3, 2) if one else (3, 2, 1)):
                        if M * max(N, K) > 32768 * 6144 // 2 and path == 1:
                            continue
                        if path == 3 and N % 256:
                            continue
                        a, b = bits((M, K)), bits((K, N) if b_mn else (N, K))
                        q8 = os.environ.get("SWEEP_Q8") == "1"
                        if q8:  # the same shape with the weight as Q8_0 blocks, dequantised in the GEMM
                            if path not in (0, 3, 5):
                                continue
                            wq = q8_0(0.02 * rng.standard_normal((K, N) if b_mn else (N, K)).astype(np.float32))
                            _, ms = A.gemm_q8_0(a, wq, M, N, K, b_mn, path, reps=reps)
                        else:
                            _, ms = A.gemm_f16(a, b, M, N, K, b_mn, path, reps=reps)
                        tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
                        print(json.dumps({"sweep": "gemm", "M": M, "N": N, "K": K,
                                          "layout": "NN (dX = dY W)" if b_mn else "NT (Y = X W^T)",
                                          "kernel": {1: "mma.sync", 2: "tcgen05", 3: "tcgen05_pair"}[path],
                                          "weights": "q8_0" if q8 else "f16", "ms": ms,
                                          "tflops": tf, "frac_of_peak": tf / peak}), flush=True)
    elif kind == "record":
        run_sweep_record(A, reps, peak)
    else:
        # cross-attention over the 32 conditioning tokens first (the tcgen05 query-major kernels of
        # xattn_tc.cu), then self-attention
        for H in (16, 24):
            for T in (750, 1500):
                clips = max(1, 6000 // T)
                D = H * 64
                q, do = bits((clips * T, D)), bits((clips * T, D))
                k, v = bits((clips * 32, D)), bits((clips * 32, D))
                A.attention(q, k, v, do, clips, T, 32, H, [32] * clips, False, True, None)  # warm
                out = A.attention(q, k, v, do, clips, T, 32, H, [32] * clips, False, True, None)
                byts_f, byts_b = 4.0 * clips * T * D, 6.0 * clips * T * D  # Q in + O out; Q, dO in + dQ out
                print(json.dumps({"sweep": "cross_attention", "heads": H, "seq": T, "keys": 32, "clips": clips,
                                  "ms_fwd": out["ms_fwd"], "ms_bwd": out["ms_bwd"],
                                  "gbs_fwd": byts_f / (out["ms_fwd"] / 1e3) / 1e9,
                                  "gbs_bwd": byts_b / (out["ms_bwd"] / 1e3) / 1e9}), flush=True)
        for H in (16, 24):
            for T in (750, 1500, 3000):
                for causal in (False, True):
                    clips = max(1, 6000 // T)
                    D = H * 64
                    q, k, v, do = (bits((clips * T, D)) for _ in range(4))
                    A.attention(q, k, v, do, clips, T, T, H, None, causal, not causal, None)  # warm
                    out = A.attention(q, k, v, do, clips, T, T, H, None, causal, not causal, None)
                    keys = T * (T + 1) / 2 if causal else T * (T + 1)
                    f_fwd, f_bwd = 4.0 * clips * keys * D, 8.0 * clips * keys * D
                    print(json.dumps({"sweep": "attention", "heads": H, "seq": T, "clips": clips, "causal": causal,
                                      "zero_key": not causal, "ms_fwd": out["ms_fwd"], "ms_bwd": out["ms_bwd"],
                                      "tflops_fwd": f_fwd / (out["ms_fwd"] / 1e3) / 1e12,
                                      "tflops_bwd": f_bwd / (out["ms_bwd"] / 1e3) / 1e12}), flush=True)


def run_sweep_record(A, reps, peak):
    """The kernel sweep of BASELINE cfg 5 as one record: the cfg-2 / cfg-4 projection shapes and
    2k-64k token rows at the cfg-2 widths with f16 and Q8_0 weights beside cuBLAS (torch.matmul,
    f16 in / f16 out, fp32 accumulation) timed in the same process; the four LoRA rank products at
    ranks 8..64 and the DoRA weight products on a Q8_0 weight; self-attention at 750 / 1500 / 3000
    frames, 16 and 24 heads, causal and not.  Every GEMM result is checked against cuBLAS's."""
    import torch
    rng = np.random.default_rng(0)
    bits = lambda shape: (rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16) ^
                          (rng.integers(0, 2, size=shape, dtype=np.uint16) << 15))
    dev = torch.device("cuda", 0)

    def cublas_ms(a16, b16, b_mn):
        x = torch.from_numpy(a16.view(np.float16)).to(dev)
        w = torch.from_numpy(b16.view(np.float16)).to(dev)
        f = (lambda: torch.matmul(x, w)) if b_mn else (lambda: torch.matmul(x, w.t()))
        for _ in range(3):
            y = f()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            f()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, y.float().cpu().numpy()

    def gemm_line(M, N, K, b_mn, part):
        wshape = (K, N) if b_mn else (N, K)
        a = bits((M, K))
        w32 = (0.02 * rng.standard_normal(wshape)).astype(np.float32)
        blocks = q8_0(w32)
        _, wh = A.q8_0_dequant(blocks)
        wh = wh.reshape(wshape)
        c16, ms16 = A.gemm_f16(a, wh, M, N, K, b_mn, 0, reps=reps)
        c8, ms8 = A.gemm_q8_0(a, blocks, M, N, K, b_mn, 0, reps=reps)
        msc, cref = cublas_ms(a, wh, b_mn)
        fl = 2.0 * M * N * K
        scale = np.abs(cref).max()
        print(json.dumps({"sweep": "gemm", "part": part, "M": M, "N": N, "K": K,
                          "layout": "NN (dX = dY W)" if b_mn else "NT (Y = X W^T)",
                          "ms_f16": ms16, "ms_q8_0": ms8, "ms_cublas": msc,
                          "tflops_f16": fl / ms16 / 1e9, "tflops_q8_0": fl / ms8 / 1e9, "tflops_cublas": fl / msc / 1e9,
                          "frac_of_peak_f16": fl / ms16 / 1e9 / peak, "frac_of_peak_q8_0": fl / ms8 / 1e9 / peak,
                          "max_rel_diff_vs_cublas": float(max(np.abs(c16 - cref).max(), np.abs(c8 - cref).max()) / scale),
                          "q8_0_equals_f16": bool(np.array_equal(c8, c16))}), flush=True)

    # the projection shapes of the benchmarked steps (cfg 2: 8 x 750 rows, cfg 4: 4 x 1 503 rows)
    shapes = [(6000, 1024, 1024), (6000, 3072, 1024), (6000, 4096, 1024), (6000, 1024, 4096),
              (6012, 1536, 1536), (6012, 4608, 1536), (6012, 6144, 1536), (6012, 1536, 6144)]
    for M, N, K in shapes:
        for b_mn in (False, True):
            gemm_line(M, N, K, b_mn, "step shapes")
    # cfg 5's token counts at the cfg-2 projection widths (forward layout)
    for M in (2048, 8192, 32768, 65536):
        for N, K in ((1024, 1024), (4096, 1024), (1024, 4096)):
            gemm_line(M, N, K, False, "token sweep")
    for K in (1024, 4096):
        for r in (8, 16, 32, 64):
            nb = (r + 31) // 32 * 32
            for kind, name, a_mn, b_mn, M, KK in ((2, "U = s X A^T", 0, 0, 6000, K), (2, "dU = s dY B", 0, 1, 6000, K),
                                                  (0, "dB += dY^T U", 1, 1, K, 6000), (1, "dA += dU^T X", 1, 1, K, 6000)):
                aa = bits((KK, M) if a_mn else (M, KK))
                bb = bits((KK, nb) if b_mn else (nb, KK))
                _, ms = A.rank_gemm_f16(aa, bb, M, KK, nb, bool(a_mn), bool(b_mn), kind, 1.0, reps=reps)
                byts = 2.0 * M * KK + 2.0 * KK * nb
                print(json.dumps({"sweep": "rank", "product": name, "rank": r, "M": M, "K": KK, "nb": nb, "ms": ms,
                                  "gbs": byts / ms / 1e6}), flush=True)
    # the DoRA weight products on a Q8_0 weight (P = W A^T, K-major; BD^T W, MN-major), cfg-4 widths
    for M, K in ((4608, 1536), (1536, 1536), (6144, 1536), (1536, 6144)):
        for kind, name, a_mn, b_mn in ((0, "P = W A^T", 0, 0), (1, "BD^T W", 1, 1)):
            mm, kk = (M, K) if not a_mn else (K, M)  # BD^T W reduces over the weight's rows
            wshape = (kk, mm) if a_mn else (mm, kk)
            blocks = q8_0((0.02 * rng.standard_normal(wshape)).astype(np.float32))
            bb = bits((kk, 32) if b_mn else (32, kk))
            _, ms = A.rank_gemm_q8_0(blocks, bb, mm, kk, 32, bool(a_mn), bool(b_mn), kind, 1.0, reps=reps)
            byts = 1.0625 * mm * kk + 2.0 * kk * 32 + 8.0 * mm * 32
            print(json.dumps({"sweep": "rank_q8_0", "product": name, "M": mm, "K": kk, "nb": 32, "ms": ms,
                              "gbs": byts / ms / 1e6}), flush=True)
    for H in (16, 24):
        for T in (750, 1500, 3000):
            for causal in (False, True):
                clips = max(1, 6000 // T)
                D = H * 64
                q, k, v, do = (bits((clips * T, D)) for _ in range(4))
                A.attention(q, k, v, do, clips, T, T, H, None, causal, not causal, None)
                out = A.attention(q, k, v, do, clips, T, T, H, None, causal, not causal, None)
                keys = T * (T + 1) / 2 if causal else T * (T + 1)
                print(json.dumps({"sweep": "attention", "heads": H, "seq": T, "clips": clips, "causal": causal,
                                  "zero_key": not causal, "ms_fwd": out["ms_fwd"], "ms_bwd": out["ms_bwd"],
                                  "tflops_fwd": 4.0 * clips * keys * D / (out["ms_fwd"] / 1e3) / 1e12,
                                  "tflops_bwd": 8.0 * clips * keys * D / (out["ms_bwd"] / 1e3) / 1e12}), flush=True)


def build_context(A, c, workload, device, seed=0):
    rng = np.random.default_rng(seed)
    if workload.startswith("mf"):
        md = A.mf_model(c["dim"], c["layers"], c["heads"], c["ff"], c["lat"], c["cond"], c["tdim"])
        ad = A.AdapterDesc(A.ADAPTER_LORA, c["rank"], c["alpha"], 0, c["targets"], 1234, c["batch"], c["T"], c["C"], 0)
        tensors = dit_tensors(c)
    else:
        md = A.mg_model(c["dim"], c["layers"], c["heads"], c["ff"], c["n_q"], c["card"])
        ad = A.AdapterDesc(A.ADAPTER_DORA_ROWS, c["rank"], c["alpha"], 0, c["targets"], 1234, c["batch"], c["frames"],
                           c["C"], 0)
        tensors = lm_tensors(c)
    ctx = A.Context(md, ad, device)
    for name, shape in tensors:
        w, kind = synth_weight(rng, name, shape)
        if kind == "q8_0" and c.get("weights") == "f16":
            ctx.bind(name, w.astype(np.float16).view(np.uint16), A.TYPE_F16)
        elif kind == "q8_0":
            ctx.bind(name, q8_0(w), A.TYPE_Q8_0)
        else:
            ctx.bind(name, w, A.TYPE_F32)
    ctx.finalize()
    return ctx


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="mf", choices=["mf", "mf-cfg1", "mg"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0, help="override depth (profiling captures only)")
    ap.add_argument("--batch", type=int, default=0, help="override clips per rank (profiling captures only)")
    ap.add_argument("--sweep", choices=["gemm", "attention", "record"], help="kernel-level sweep instead of the step")
    args = ap.parse_args()
    if args.sweep:
        return run_sweep(args.sweep, max(args.steps, 3))
    c = dict({"mf": MF, "mf-cfg1": MF1, "mg": MG}[args.workload])
    if args.layers:
        c["layers"] = args.layers
    if args.batch:
        c["batch"] = args.batch
    if args.impl == "reference":
        return run_reference(args, c)

    import torch
    import torch.distributed as dist
    import actrain as A

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    host = None
    if world > 1:
        from datetime import timedelta
        import dp
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        host = dp.host_group(120.0)  # host-side coordination (gloo), bounded

    ctx = build_context(A, c, args.workload, local)
    if world > 1:
        ctx.set_timeout(120_000)  # a stalled peer ends in an aborted communicator, not a hang
        ctx.nccl_init(dp.share_nccl_id(host, rank, A.Context.nccl_unique_id), world, rank)

    rng = np.random.default_rng(1000 + rank)
    n = c["batch"]
    if args.workload.startswith("mf"):
        batch = (rng.standard_normal((n, c["lat"], c["T"]), dtype=np.float32),
                 rng.standard_normal((n, c["lat"], c["T"]), dtype=np.float32),
                 rng.standard_normal((n, c["C"], c["cond"]), dtype=np.float32),
                 rng.uniform(0, 1, n).astype(np.float32), np.zeros(n, np.int32), np.full(n, -1, np.int32))
        stage = lambda: ctx.mf_stage(*batch)
        e2e_step = lambda: ctx.mf_step(*batch)
        h2d = sum(a.nbytes for a in batch[:4]) + 4 * n * (1 + c["tdim"])
    else:
        batch = (rng.integers(0, c["card"], (n, c["n_q"], c["frames"])).astype(np.int32),
                 rng.standard_normal((n, c["C"], c["dim"]), dtype=np.float32))
        stage = lambda: ctx.mg_stage(*batch)
        e2e_step = lambda: ctx.mg_step(*batch)
        T = c["frames"] + c["n_q"] - 1
        h2d = n * c["n_q"] * (T + c["frames"]) * 4 + batch[1].nbytes
    d2h = 4 * n

    stream = torch.cuda.ExternalStream(ctx.stream())
    step_counter = [0]

    def one_step(e2e=False):
        if world > 1:  # the step all-reduces its gradients itself, layer by layer, overlapping the backward
            ctx.set_grad_sync(n * world)
        if e2e:
            e2e_step()
        else:
            ctx.run_staged(n, read_loss=False)
        step_counter[0] += 1
        ctx.optimizer(lr=1e-4, step=step_counter[0], weight_decay=0.01, clip=1.0)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- warm-up (first call runs eagerly, second captures the CUDA graph)
    stage()
    for _ in range(max(args.warmup, 3)):
        one_step()
    barrier()
    if host is not None:  # every rank is alive and through its warm-up before anything is timed
        dp.check_peers(host, 120.0, "the timed steps")

    # ---- value: device-timed, inputs resident in HBM
    clocks = Clocks(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for _ in range(args.steps):
        one_step()
    ev1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_per_step = ms / args.steps
    value = world * args.steps / (ms / 1e3)

    # ---- e2e: through the public API with host buffers (H2D inputs + D2H losses inside)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step(e2e=True)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = world * args.steps / e2e_s

    # ---- kernel classes from eagerly launched, event-bracketed steps (profiling mode)
    ctx.set_profiling(True)
    ctx.reset_kernel_stats()
    stage()
    for _ in range(2):
        one_step()
    ctx.set_profiling(False)
    stats = [ctx.kernel_stats(i) for i in range(3)]
    kernels_per_step = ctx.graph_kernel_nodes(n) + 2
    step_flops = ctx.step_flops(n)

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    peak_tf = peaks.get("bf16_tflops_sustained", 1400.0)
    peak_src = "measured (sustained)" if "bf16_tflops_sustained" in peaks else "fallback (sustained)"
    g = stats[0]
    achieved = g["flops"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
    traffic = None
    try:
        prof = json.load(open(os.path.join(ROOT, "profiles", "gemm_traffic.json")))
        # the capture covers one workload's shapes; another workload's launches move other bytes
        if prof.get("bench_workload") == args.workload:
            traffic = prof.get("bytes_per_launch")
    except (OSError, ValueError):
        pass

    metric, line_unit, config = line_header(args, c, n, world)
    line = {
        "metric": metric,
        "value": value, "unit": line_unit,
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": config,
        "e2e": {"value": e2e_value, "unit": line_unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": int(kernels_per_step * args.steps),
        "step_tflops": step_flops / (ms_per_step / 1e3) / 1e12,
        "step_frac_of_peak": step_flops / (ms_per_step / 1e3) / 1e12 / peak_tf,
        "roofline": {"kernel": "dense projection GEMMs (class 0)", "bound": "tensor", "achieved": achieved,
                     "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf if peak_tf else None,
                     "traffic": traffic, "peak_source": peak_src,
                     "launches_per_step": g["launches"] / 2, "ms_per_step": g["ms"] / 2},
        "kernel_classes_ms_per_step": {"gemm": stats[0]["ms"] / 2, "attention": stats[1]["ms"] / 2,
                                       "other": stats[2]["ms"] / 2},
    }
    if clk:
        line["clocks"] = clk
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        dt, scale, desc = cpu_sample(c)
        line["cpu_baseline"] = {"value": 1.0 / (dt * scale), "unit": line_unit, "cores": os.cpu_count(),
                                "kind": "port", "sample": desc, "sample_seconds": dt, "sample_scale": scale}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
