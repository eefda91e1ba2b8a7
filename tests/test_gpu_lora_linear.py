"""Adapter consumption on the GPU (act_lora_linear): inference lora_linear of src/ac/lora.h:50-83
with the scale and strength rules of load_lora (src/ac/lora.h:113-170), against an fp64 numpy
restatement on the same f16-rounded operands the tensor cores see.  F32, F16 and Q8_0 weights,
LoRA and DoRA rows, strength 1 / 0.4 / 0, rows below and above the 2-CTA kernel's minimum."""
import numpy as np
import pytest

import actrain as A
from cases import q8_0_bytes
from f16util import f16_bits, bits_to_f32

pytestmark = pytest.mark.gpu


def reference(x, W, Am, Bm, alpha, m, strength):
    """lora_linear in fp64 (x and W as the device rounds them)."""
    x64, W64 = x.astype(np.float64), W.astype(np.float64)
    base = x64 @ W64.T
    if Am is None:
        return base
    A64, B64 = Am.astype(np.float64), Bm.astype(np.float64)
    r = A64.shape[0]
    ba = (x.astype(np.float64) @ A64.T) @ B64.T
    if m is None:
        return base + strength * alpha / r * ba
    s = alpha / r
    if strength == 0:
        return base
    nsq = (W64 ** 2).sum(1) + W.shape[1] * 1e-12 + 2 * s * ((W64 @ A64.T) * B64).sum(1) + \
        s * s * ((B64 @ (A64 @ A64.T)) * B64).sum(1)
    y = (base + s * ba) * (m.astype(np.float64) / np.sqrt(nsq))
    return base + strength * (y - base)


@pytest.mark.parametrize("wtype", ["f32", "f16", "q8_0"])
@pytest.mark.parametrize("dora", [False, True], ids=["lora", "dora"])
@pytest.mark.parametrize("strength", [1.0, 0.4, 0.0])
@pytest.mark.parametrize("rows", [96, 700])
def test_lora_linear_matches_the_restatement(wtype, dora, strength, rows):
    rng = np.random.default_rng(rows + 7 * int(dora) + int(10 * strength))
    n_in, out, r, alpha = 256, 384, 8, 16.0
    x = rng.standard_normal((rows, n_in)).astype(np.float32)
    Wf = (0.05 * rng.standard_normal((out, n_in))).astype(np.float32)
    Am = (0.1 * rng.standard_normal((r, n_in))).astype(np.float32)
    Bm = (0.1 * rng.standard_normal((out, r))).astype(np.float32)
    m = (np.sqrt((Wf ** 2).sum(1)) * (1 + 0.1 * rng.standard_normal(out))).astype(np.float32) if dora else None
    if wtype == "f32":
        raw, t, Wdev = Wf, A.TYPE_F32, bits_to_f32(f16_bits(Wf)).reshape(Wf.shape)
        Wnorm = Wf
    elif wtype == "f16":
        h = Wf.astype(np.float16)
        raw, t, Wdev = h.view(np.uint16), A.TYPE_F16, h.astype(np.float32)
        Wnorm = Wdev
    else:
        raw = q8_0_bytes(Wf)
        f32, h16 = A.q8_0_dequant(raw)
        raw, t, Wdev, Wnorm = raw, A.TYPE_Q8_0, bits_to_f32(h16).reshape(Wf.shape), f32.reshape(Wf.shape)
    xd = bits_to_f32(f16_bits(x)).reshape(x.shape)
    y = A.lora_linear(x, raw, t, out, Am, Bm, alpha, m, strength)
    # the base on the device operands; the adapter path and the norms on the stored fp32 values
    base = xd.astype(np.float64) @ Wdev.astype(np.float64).T
    full = reference(x, Wnorm, Am, Bm, alpha, m, strength)
    ref = base + (full - x.astype(np.float64) @ Wnorm.astype(np.float64).T) if not dora or strength == 0 else None
    if dora and strength != 0:
        # DoRA scales the base too: y = base + strength (g (base + s BAx) - base), g from fp32 norms
        r_ = Am.shape[0]
        s = alpha / r_
        ba = (x.astype(np.float64) @ Am.astype(np.float64).T) @ Bm.astype(np.float64).T
        W64, A64, B64 = Wnorm.astype(np.float64), Am.astype(np.float64), Bm.astype(np.float64)
        nsq = (W64 ** 2).sum(1) + n_in * 1e-12 + 2 * s * ((W64 @ A64.T) * B64).sum(1) + \
            s * s * ((B64 @ (A64 @ A64.T)) * B64).sum(1)
        yd = (base + s * ba) * (m / np.sqrt(nsq))
        ref = base + strength * (yd - base)
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err < 2e-5, err


def test_bare_projection_and_bad_arguments():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((300, 128)).astype(np.float32)
    W = (0.05 * rng.standard_normal((64, 128))).astype(np.float32)
    y = A.lora_linear(x, W, A.TYPE_F32, 64)
    ref = bits_to_f32(f16_bits(x)).reshape(x.shape).astype(np.float64) @ \
        bits_to_f32(f16_bits(W)).reshape(W.shape).astype(np.float64).T
    assert np.abs(y - ref).max() / np.abs(ref).max() < 2e-5
    with pytest.raises(A.ActError):  # rank above the supported 64
        A.lora_linear(x, W, A.TYPE_F32, 64, np.zeros((65, 128), np.float32), np.zeros((64, 65), np.float32), 1.0)
    with pytest.raises(A.ActError):  # weight bytes disagree with [out][in]
        A.lora_linear(x, W[:32], A.TYPE_F32, 64)
