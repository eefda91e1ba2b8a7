"""Pins for the CPU oracle (no GPU).

Each test names the reference test or file it mirrors (paths in the audiocraft.cpp tree).
"""
import ctypes as C
import json
import os

import numpy as np
import pytest

import oracle as O
from fixtures import GOLDEN, fixture_paths, load


# ---------------------------------------------------------------------------------------
# the fp64 autograd restatement (tests/golden/gen_fixtures.py) vs the C oracle

@pytest.mark.parametrize("path", fixture_paths("dit") + fixture_paths("lm"),
                         ids=lambda p: os.path.basename(p))
def test_oracle_matches_fp64_autograd_fixture(path):
    z, c, ad = load(path)
    if str(z["kind"]) == "dit":
        loss, g = O.dit_step(c, z["W"], ad, z["params"], z["clean"], z["noise"], z["hidden"],
                             z["t"], z["uncond"], z["valid"])
    else:
        loss, g = O.lm_step(c, z["W"], ad, z["params"], z["codes"], z["context"], int(z["prefix"]))
    np.testing.assert_allclose(loss, z["loss"], rtol=2e-6)
    ref = z["grads"]
    rel = np.linalg.norm(g - ref) / max(np.linalg.norm(ref), 1e-30)
    assert rel < 5e-6, rel
    np.testing.assert_allclose(g, ref, rtol=1e-3, atol=1e-6 * np.abs(ref).max())


# ---------------------------------------------------------------------------------------
# Q8_0 (gguf-py goldens, bit exact)

def test_q8_0_dequant_and_quant_bit_exact():
    z = np.load(os.path.join(GOLDEN, "q8_0.npz"))
    x, q, deq = z["x"], z["q"], z["deq"]
    out = np.zeros(x.size, np.float32)
    O.lib().ora_q8_0_dequant(np.ascontiguousarray(q.ravel()), x.shape[0], out)
    assert np.array_equal(out.view(np.uint32), deq.ravel().view(np.uint32))
    qq = np.zeros(q.size, np.uint8)
    O.lib().ora_q8_0_quant(np.ascontiguousarray(x.ravel()), x.shape[0], qq)
    assert np.array_equal(qq, q.ravel())


def test_half_conversion_roundtrip():
    L = O.lib()
    h = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([L.ora_half_to_float(int(v)) for v in h[::97]], np.float32)
    sel = ref[::97]
    finite = np.isfinite(sel)
    assert np.array_equal(got[finite], sel[finite])
    xs = np.random.default_rng(0).standard_normal(4000).astype(np.float32) * 10.0 ** \
        np.random.default_rng(1).uniform(-9, 5, 4000).astype(np.float32)
    back = np.array([L.ora_float_to_half(float(v)) for v in xs], np.uint16)
    assert np.array_equal(back, xs.astype(np.float16).view(np.uint16))


# ---------------------------------------------------------------------------------------
# delay pattern goldens (tests/pattern_test.cpp:93-146)

def test_delay_pattern_goldens():
    cases = json.load(open(os.path.join(GOLDEN, "pattern_goldens.json")))["cases"]
    L = O.lib()
    for tag, c in cases.items():
        nq, T, S, sp = c["n_q"], c["T"], c["S"], c["special"]
        codes = np.array(c["codes"], np.int32)
        seq = np.zeros(nq * S, np.int32)
        L.ora_pattern_build(nq, T, codes, sp, seq)
        assert seq.tolist() == c["sequence"], tag
        rev = np.zeros(nq * T, np.int32)
        L.ora_pattern_revert(nq, T, seq, sp, rev)
        assert rev.tolist() == c["reverted"], tag
        mask = np.zeros(nq * S, np.uint8)
        L.ora_pattern_mask(nq, T, mask)
        assert mask.tolist() == c["mask"], tag


def test_pattern_generation_shape():
    # tests/pattern_test.cpp: 1500 timesteps, 4 codebooks -> 1504 steps.
    nq, T = 4, 1500
    codes = np.arange(nq * T, dtype=np.int32)
    seq = np.zeros(nq * (T + nq), np.int32)
    O.lib().ora_pattern_build(nq, T, codes, 2048, seq)
    seq = seq.reshape(nq, T + nq)
    for q in range(nq):
        assert (seq[q, 1 + q:1 + q + T] == codes[q * T:(q + 1) * T]).all()
        assert (seq[q, :1 + q] == 2048).all() and (seq[q, 1 + q + T:] == 2048).all()


# ---------------------------------------------------------------------------------------
# U-ViT skip plan (tests/dit_skip_test.cpp:95-130)

def _plan(idx, L, n):
    c, p, j = C.c_int(), C.c_int(), C.c_int()
    O.lib().ora_skip_plan(idx, L, n, C.byref(c), C.byref(p), C.byref(j))
    return c.value, p.value, j.value


def test_skip_projection_order_24_layers():
    got = [_plan(i, 24, 11)[2] for i in range(24) if _plan(i, 24, 11)[0]]
    assert got == [2, 3, 4, 5, 6, 7, 8, 9, 10, 0, 1]
    assert [i for i in range(24) if _plan(i, 24, 11)[1]] == list(range(11))


@pytest.mark.parametrize("layers", range(4, 34))
def test_skip_stack_drains(layers):
    n = (layers - 1) // 2
    depth = 0
    for i in range(layers):
        c, p, _ = _plan(i, layers, n)
        if c:
            assert depth > 0
            depth -= 1
        if p:
            depth += 1
    assert depth == 0


# ---------------------------------------------------------------------------------------
# optimizer (tests/train_controls_test.cpp:6-33)

def test_optimizer_golden():
    L = O.lib()
    assert L.ora_rate(1.0, 1, 4, 0) == np.float32(0.25)
    assert L.ora_rate(1.0, 4, 4, 0) == 1.0 and L.ora_rate(1.0, 5, 4, 0) == 1.0
    value = np.array([2.0, 2.0], np.float32)
    m = np.zeros(2, np.float32)
    v = np.zeros(2, np.float32)
    grad = np.array([6.0, 8.0], np.float32)        # sums over count = 2
    decays = np.array([1, 0], np.uint8)            # lora_A decays, magnitude does not
    bad = L.ora_adamw(2, value, m, v, grad, decays, 2, 1, 0.1, 0.0, 0.0, 1e-8, 0.1, 1.0)
    assert bad == 0
    assert abs(m[0] - 0.6) < 1e-6 and abs(m[1] - 0.8) < 1e-6
    assert abs(value[0] - 1.88) < 1e-6 and abs(value[1] - 1.9) < 1e-6


# ---------------------------------------------------------------------------------------
# gradient invariants of tests/mf_lora_test.cpp on the oracle

def _tiny():
    z, c, ad = load(os.path.join(GOLDEN, "dit_tiny_lora.npz"))
    return z, c, ad


def test_gelu_gradient_finite_difference():
    L = O.lib()
    for x in np.linspace(-4, 4, 41):
        if abs(x) < 1e-3:
            continue
        fd = (L.ora_gelu(x + 1e-3) - L.ora_gelu(x - 1e-3)) / 2e-3
        assert abs(L.ora_gelu_grad(x) - fd) < 2e-3


def test_zero_b_gives_zero_a_gradient():
    z, c, ad = load(os.path.join(GOLDEN, "dit_tiny_lora_zeroB.npz"))
    _, g = O.dit_step(c, z["W"], ad, z["params"], z["clean"], z["noise"], z["hidden"], z["t"],
                      z["uncond"], z["valid"])
    lay = O.adapter_layout(c.dim, c.ff_dim, c.layers, ad)
    for name, off, shape in lay:
        n = int(np.prod(shape))
        if name.endswith("lora_A"):
            assert np.all(np.abs(g[off:off + n]) < 1e-8), name
    assert np.any(np.abs(g) > 1e-6)


@pytest.mark.parametrize("name", ["dit_tiny_lora.npz", "dit_tiny_dora.npz", "dit_small_dora.npz"])
def test_finite_difference_adapter_gradients(name):
    z, c, ad = load(os.path.join(GOLDEN, name))
    params = z["params"].copy()
    loss0, g = O.dit_step(c, z["W"], ad, params, z["clean"], z["noise"], z["hidden"], z["t"],
                          z["uncond"], z["valid"])
    lay = O.adapter_layout(c.dim, c.ff_dim, c.layers, ad)
    picks = [lay[0], lay[1], lay[2], lay[-1]]
    for nm, off, shape in picks:
        n = int(np.prod(shape))
        k = off + int(np.argmax(np.abs(g[off:off + n])))
        eps = 0.002
        saved = params[k]
        params[k] = saved + eps
        lp, _ = O.dit_step(c, z["W"], ad, params, z["clean"], z["noise"], z["hidden"], z["t"],
                           z["uncond"], z["valid"], grads=False)
        params[k] = saved - eps
        lm, _ = O.dit_step(c, z["W"], ad, params, z["clean"], z["noise"], z["hidden"], z["t"],
                           z["uncond"], z["valid"], grads=False)
        params[k] = saved
        fd = (lp.sum() - lm.sum()) / (2 * eps)
        assert abs(g[k] - fd) < 2e-4 + 0.03 * abs(fd), (nm, g[k], fd)


def test_adam_steps_reduce_tiny_loss():
    # tests/mf_lora_test.cpp:195-198: 30 Adam steps (lr 0.004) bring the loss below 0.9x.
    z, c, ad = _tiny()
    params = z["params"].copy()
    lay = O.adapter_layout(c.dim, c.ff_dim, c.layers, ad)
    decays = np.zeros(params.size, np.uint8)
    m = np.zeros_like(params)
    v = np.zeros_like(params)
    args = (z["clean"][:1], z["noise"][:1], z["hidden"][:1], z["t"][:1], z["uncond"][:1],
            z["valid"][:1])
    before, _ = O.dit_step(c, z["W"], ad, params, *args, grads=False)
    for step in range(1, 31):
        _, g = O.dit_step(c, z["W"], ad, params, *args)
        O.lib().ora_adamw(params.size, params, m, v, g, decays, 1, step, 0.004, 0.9, 0.999,
                          1e-8, 0.0, 1.0)
    after, _ = O.dit_step(c, z["W"], ad, params, *args, grads=False)
    assert after[0] < 0.9 * before[0]
    assert len(lay) > 0


def test_unconditional_cross_attention_gets_no_gradient():
    # tests/mf_train_torch_parity.py:160-161: masked cross-attention receives no gradient.
    z, c, ad = load(os.path.join(GOLDEN, "dit_small_lora.npz"))
    sel = np.array([2])   # the unconditional clip
    _, g = O.dit_step(c, z["W"], ad, z["params"], z["clean"][sel], z["noise"][sel],
                      z["hidden"][sel], z["t"][sel], z["uncond"][sel], z["valid"][sel])
    for name, off, shape in O.adapter_layout(c.dim, c.ff_dim, c.layers, ad):
        n = int(np.prod(shape))
        if ".cross." in name:
            assert np.count_nonzero(g[off:off + n]) == 0, name
