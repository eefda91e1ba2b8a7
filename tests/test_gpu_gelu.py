"""The feed-forward activation on bf16 inputs: the lookup table the training step uses equals the
direct A&S evaluation (src/ac/lora.h:97-110 and its derivative) bit for bit on every finite bf16
value below 2^127, and both agree with the oracle's fp32 restatement to one bf16 unit in the last
place.  At the top exponent (|z| >= 2^127) the direct derivative overflows (2|z| is infinite and
multiplies a zero exponential); there the table keeps the limits gelu = z (or -0), gelu' = 1 (or -0)."""
import os
import sys

import numpy as np
import pytest

import actrain as A

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))


def all_finite_bf16(top=False):
    z = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    e = (z >> 7) & 0xFF
    return z[e == 0xFE] if top else z[e < 0xFE]


def bits_to_f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def ordered(b):  # bf16 bits -> integers ordered like the values (+0 and -0 coincide)
    b = b.astype(np.int64)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def test_table_equals_direct_evaluation():
    z = all_finite_bf16()
    g_t, d_t = A.gelu_bf16(z, direct=False)
    g_d, d_d = A.gelu_bf16(z, direct=True)
    np.testing.assert_array_equal(ordered(g_t), ordered(g_d))
    np.testing.assert_array_equal(ordered(d_t), ordered(d_d))


def test_table_limits_at_the_top_exponent():
    z = all_finite_bf16(top=True)
    g, d = A.gelu_bf16(z, direct=False)
    neg = (z >> 15) == 1
    np.testing.assert_array_equal(g[~neg], z[~neg])
    np.testing.assert_array_equal(d[~neg], np.full((~neg).sum(), 0x3F80, np.uint16))
    assert np.all(ordered(g[neg]) == 0) and np.all(ordered(d[neg]) == 0)


def test_direct_matches_oracle_within_one_ulp():
    import oracle as O
    L = O.lib()
    z = all_finite_bf16()
    zf = bits_to_f32(z)
    g_o = f32_to_bf16_bits(np.array([L.ora_gelu(float(v)) for v in zf], np.float32))
    d_o = f32_to_bf16_bits(np.array([L.ora_gelu_grad(float(v)) for v in zf], np.float32))
    g_d, d_d = A.gelu_bf16(z, direct=True)
    for got, ref in ((g_d, g_o), (d_d, d_o)):
        diff = np.abs(ordered(got) - ordered(ref))
        assert diff.max() <= 1, diff.max()
        assert np.mean(diff > 0) < 0.02
