"""Attention kernels (act_attention) vs an fp64 numpy restatement of src/ac/transformer.h:108-125
(dense softmax with the optional zero key and additive masks) with the stored-frequency RoPE of
src/ac/transformer.h:55-61.  Tolerance: relative L2 <= 1e-2 per output (f16 operands)."""
import numpy as np
import pytest

import actrain as A
from f16util import bits_to_f32, f16_bits

pytestmark = pytest.mark.gpu


def f32(b):
    return bits_to_f32(b).astype(np.float64)


def rope_table(T):
    ff = 10000.0 ** (2 * np.arange(32) / 64.0)
    th = (np.arange(T, dtype=np.float32)[:, None] / ff[None, :].astype(np.float32)).astype(np.float32)
    return np.stack([np.cos(th), np.sin(th)], -1).astype(np.float32)  # [T][32][2]


def rotate(x, tab, inverse=False):
    T = x.shape[0]
    c, s = tab[:T, :, 0].astype(np.float64), tab[:T, :, 1].astype(np.float64)
    if inverse:
        s = -s
    y = x.reshape(T, -1, 32, 2).copy()
    x0, x1 = y[..., 0].copy(), y[..., 1].copy()
    y[..., 0] = x0 * c[:, None, :] - x1 * s[:, None, :]
    y[..., 1] = x0 * s[:, None, :] + x1 * c[:, None, :]
    return y.reshape(x.shape)


def reference(q, k, v, do, clips, T, Tk, H, nvalid, causal, zero_key, tab):
    D = H * 64
    o = np.zeros((clips * T, D)); dq = np.zeros_like(o); dk = np.zeros((clips * Tk, D)); dv = np.zeros_like(dk)
    for b in range(clips):
        Q, K, V, dO = q[b * T:(b + 1) * T], k[b * Tk:(b + 1) * Tk], v[b * Tk:(b + 1) * Tk], do[b * T:(b + 1) * T]
        if tab is not None:
            Q, K = rotate(Q, tab), rotate(K, tab)
        nv = Tk if nvalid is None else min(Tk, nvalid[b])
        for h in range(H):
            sl = slice(h * 64, (h + 1) * 64)
            s = Q[:, sl] @ K[:, sl].T / 8.0
            mask = np.zeros_like(s, bool)
            mask[:, nv:] = True
            if causal:
                mask |= np.triu(np.ones_like(mask), 1)
            s[mask] = -np.inf
            if zero_key:
                s = np.concatenate([np.zeros((T, 1)), s], 1)
            m = s.max(1, keepdims=True)
            p = np.exp(s - m)
            p /= p.sum(1, keepdims=True)
            pr = p[:, 1:] if zero_key else p
            oh = pr @ V[:, sl]
            o[b * T:(b + 1) * T, sl] = oh
            dpr = dO[:, sl] @ V[:, sl].T
            Dv = (dO[:, sl] * oh).sum(1, keepdims=True)
            ds = pr * (dpr - Dv)
            dqh = ds @ K[:, sl] / 8.0
            dkh = ds.T @ Q[:, sl] / 8.0
            dv[b * Tk:(b + 1) * Tk, sl] = pr.T @ dO[:, sl]
            dq[b * T:(b + 1) * T, sl] = dqh
            dk[b * Tk:(b + 1) * Tk, sl] = dkh
        if tab is not None:
            dq[b * T:(b + 1) * T] = rotate(dq[b * T:(b + 1) * T], tab, inverse=True)
            dk[b * Tk:(b + 1) * Tk] = rotate(dk[b * Tk:(b + 1) * Tk], tab, inverse=True)
    return o, dq, dk, dv


CASES = {
    "self_zero_key_rope": dict(clips=2, T=150, Tk=150, H=2, nvalid=None, causal=False, zero_key=True, rope=True),
    "cross_masked": dict(clips=3, T=90, Tk=16, H=2, nvalid=[16, 5, 0], causal=False, zero_key=True, rope=False),
    "causal": dict(clips=2, T=130, Tk=130, H=3, nvalid=None, causal=True, zero_key=False, rope=False),
    # pre-rotated inputs at the benchmark's clip length: the tcgen05 forward
    "self_zero_key_750": dict(clips=2, T=750, Tk=750, H=2, nvalid=None, causal=False, zero_key=True, rope=False),
    "causal_333": dict(clips=1, T=333, Tk=333, H=2, nvalid=None, causal=True, zero_key=False, rope=False),
    # at most 64 keys: the query-major tcgen05 cross-attention (xattn_tc.cu), with a partial last
    # query block, per-clip valid counts, with and without the zero key
    "cross_750": dict(clips=2, T=750, Tk=32, H=3, nvalid=[32, 20], causal=False, zero_key=True, rope=False),
    "cross_no_zero_key": dict(clips=3, T=200, Tk=40, H=2, nvalid=[40, 13, 1], causal=False, zero_key=False,
                              rope=False),
    "cross_64_keys": dict(clips=2, T=129, Tk=64, H=2, nvalid=None, causal=False, zero_key=True, rope=False),
}


@pytest.mark.parametrize("name", list(CASES))
def test_attention_matches_reference(name):
    c = CASES[name]
    rng = np.random.default_rng(len(name))
    D = c["H"] * 64
    q = f16_bits(rng.standard_normal((c["clips"] * c["T"], D)))
    k = f16_bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    v = f16_bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    do = f16_bits(rng.standard_normal((c["clips"] * c["T"], D)))
    tab = rope_table(c["T"]) if c["rope"] else None
    out = A.attention(q, k, v, do, c["clips"], c["T"], c["Tk"], c["H"], c["nvalid"], c["causal"], c["zero_key"], tab)
    ro, rdq, rdk, rdv = reference(f32(q), f32(k), f32(v), f32(do), c["clips"], c["T"], c["Tk"], c["H"],
                                  c["nvalid"], c["causal"], c["zero_key"], tab)
    for key, ref in (("o", ro), ("dq", rdq), ("dk", rdk), ("dv", rdv)):
        got = f32(out[key])
        scale = np.linalg.norm(ref)
        if scale == 0:
            assert np.count_nonzero(got) == 0, key
            continue
        assert np.linalg.norm(got - ref) / scale < 1e-2, (key, np.linalg.norm(got - ref) / scale)


@pytest.mark.parametrize("name", ["cross_masked", "cross_750", "cross_no_zero_key"])
def test_cross_attention_tc_matches_mma_path(name, monkeypatch):
    # the tcgen05 cross-attention against the mma.sync kernels on the same inputs (ACTRAIN_ATTN_MMA
    # routes act_attention to the latter): both restate the same softmax, so they agree to f16
    # rounding, and the log-sum-exp the forward leaves for other callers is the same
    c = CASES[name]
    rng = np.random.default_rng(7 + len(name))
    D = c["H"] * 64
    q = f16_bits(rng.standard_normal((c["clips"] * c["T"], D)))
    k = f16_bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    v = f16_bits(rng.standard_normal((c["clips"] * c["Tk"], D)))
    do = f16_bits(rng.standard_normal((c["clips"] * c["T"], D)))
    args = (q, k, v, do, c["clips"], c["T"], c["Tk"], c["H"], c["nvalid"], False, c["zero_key"], None)
    tc = A.attention(*args)
    monkeypatch.setenv("ACTRAIN_ATTN_MMA", "1")
    mma = A.attention(*args)
    for key in ("o", "dq", "dk", "dv"):
        a, b = f32(tc[key]), f32(mma[key])
        scale = np.linalg.norm(b)
        assert (np.linalg.norm(a - b) / scale if scale else np.abs(a).max()) < 5e-3, key
    fin = np.isfinite(mma["lse"])
    np.testing.assert_array_equal(fin, np.isfinite(tc["lse"]))
    np.testing.assert_allclose(tc["lse"][fin], mma["lse"][fin], rtol=0, atol=1e-4)
