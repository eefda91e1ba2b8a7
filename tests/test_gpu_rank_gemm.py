"""Rank-block products (the LoRA U, dU, dB and dA GEMMs) on the tcgen05 skinny kernel vs numpy.

f16 inputs are exact in fp32 and the kernel accumulates in fp32, so the accumulate kinds match a
float64 product to accumulation-order rounding; the f16 kind matches it to one f16 rounding.
"""
import numpy as np
import pytest

import actrain as A
from f16util import bits_to_f32, f16_bits

pytestmark = pytest.mark.gpu


def bits_to_f64(b):
    return bits_to_f32(b).astype(np.float64)


def operands(rng, M, K, nb, a_mn, b_mn):
    a = f16_bits(rng.standard_normal((K, M) if a_mn else (M, K)))
    b = f16_bits(rng.standard_normal((K, nb) if b_mn else (nb, K)))
    af = bits_to_f64(a)
    bf = bits_to_f64(b)
    Am = af.T if a_mn else af          # [M][K]
    Bm = bf if b_mn else bf.T          # [K][nb]
    return a, b, Am @ Bm


# the four products of a LoRA projection at the benchmark's sizes, plus ragged edges
CASES = [
    # (M, K, nb, a_mn, b_mn, kind)          what it is
    (6000, 1024, 32, False, False, A.RANK_STORE),   # U  = s X A^T
    (6000, 4096, 32, False, True, A.RANK_STORE),    # dU = s dY B
    (3072, 6000, 16, True, True, A.RANK_ACC),       # dB += dY^T U
    (1024, 6000, 16, True, True, A.RANK_ACC_T),     # dA += (dU^T X), stored [r][in]
    (200, 192, 64, False, False, A.RANK_STORE),     # ragged rows, full 64 columns
    (136, 100, 8, True, True, A.RANK_ACC),          # reduction tail shorter than one k-block
    (257, 4160, 24, False, True, A.RANK_ACC_T),
]


@pytest.mark.parametrize("M,K,nb,a_mn,b_mn,kind", CASES)
@pytest.mark.parametrize("splits", [0, 1], ids=["auto_split", "one_split"])
def test_rank_gemm_matches_numpy(M, K, nb, a_mn, b_mn, kind, splits):
    rng = np.random.default_rng(M * 7 + K + nb)
    a, b, ref = operands(rng, M, K, nb, a_mn, b_mn)
    alpha = 0.5
    ref = alpha * ref
    init = None
    if kind != A.RANK_STORE:
        init = rng.standard_normal((nb, M) if kind == A.RANK_ACC_T else (M, nb)).astype(np.float32)
    c = A.rank_gemm_f16(a, b, M, K, nb, a_mn, b_mn, kind, alpha, C_init=init, splits=splits)
    if kind == A.RANK_STORE:
        # one f16 rounding, plus fp32 accumulation-order error that grows like sqrt(K)
        np.testing.assert_allclose(c, ref, rtol=2 ** -11, atol=3e-5 * np.sqrt(K))
    else:
        want = init.astype(np.float64) + (ref.T if kind == A.RANK_ACC_T else ref)
        np.testing.assert_allclose(c, want, rtol=1e-5, atol=1e-5 * np.sqrt(K))


def test_rank_store_repeatable():
    # the cluster reduction sums the split-K partials in a fixed order: repeated calls agree bit for bit
    rng = np.random.default_rng(5)
    a, b, ref = operands(rng, 1000, 2048, 32, False, False)
    first = A.rank_gemm_f16(a, b, 1000, 2048, 32, False, False, A.RANK_STORE, 1.0, reps=3)[0]
    again = A.rank_gemm_f16(a, b, 1000, 2048, 32, False, False, A.RANK_STORE, 1.0)
    np.testing.assert_array_equal(first, again)
    np.testing.assert_allclose(first, ref, rtol=2 ** -11, atol=3e-5 * np.sqrt(2048))
