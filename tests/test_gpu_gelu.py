"""The feed-forward activation on f16 inputs: the vectorised pass the training step runs equals the
element-by-element A&S evaluation (src/ac/lora.h:97-110 and its derivative) bit for bit on every
finite f16 value, and both agree with the oracle's fp32 restatement to one f16 unit in the last
place."""
import os
import sys

import numpy as np
import pytest

import actrain as A
from f16util import bits_to_f32

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))


def all_finite_f16():
    z = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    return z[((z >> 10) & 0x1F) != 0x1F]


def ordered(b):  # f16 bits -> integers ordered like the values (+0 and -0 coincide)
    b = b.astype(np.int64)
    return np.where(b & 0x8000, -(b & 0x7FFF), b)


def f16_of(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def test_step_pass_equals_direct_evaluation():
    z = all_finite_f16()
    g_t, d_t = A.gelu_f16(z, direct=False)
    g_d, d_d = A.gelu_f16(z, direct=True)
    np.testing.assert_array_equal(ordered(g_t), ordered(g_d))
    np.testing.assert_array_equal(ordered(d_t), ordered(d_d))


def test_large_inputs_reach_the_limits():
    # from |z| = 16 up the A&S exponential underflows: gelu = z (or -0), gelu' = 1 (or -0)
    z = f16_of([16.0, 100.0, 65504.0, -16.0, -65504.0])
    g, d = A.gelu_f16(z, direct=False)
    np.testing.assert_array_equal(bits_to_f32(g), np.array([16.0, 100.0, 65504.0, -0.0, -0.0], np.float32))
    np.testing.assert_array_equal(bits_to_f32(d), np.array([1.0, 1.0, 1.0, -0.0, -0.0], np.float32))


def test_direct_matches_oracle_within_one_ulp():
    import oracle as O
    L = O.lib()
    z = all_finite_f16()
    zf = bits_to_f32(z)
    g_o = f16_of(np.array([L.ora_gelu(float(v)) for v in zf], np.float32))
    d_o = f16_of(np.array([L.ora_gelu_grad(float(v)) for v in zf], np.float32))
    g_d, d_d = A.gelu_f16(z, direct=True)
    for got, ref in ((g_d, g_o), (d_d, d_o)):
        diff = np.abs(ordered(got) - ordered(ref))
        assert diff.max() <= 1, diff.max()
        assert np.mean(diff > 0) < 0.02
