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


@pytest.mark.parametrize("kind,a_mn,b_mn", [(A.RANK_ACC, False, False), (A.RANK_ACC_T, True, True)],
                         ids=["P=W_At(K-major W)", "BDt_W(MN-major W)"])
@pytest.mark.parametrize("M,K,nb,splits", [(384, 1536, 32, 4), (4608, 1536, 32, 8), (1536, 6144, 16, 8),
                                           (224, 320, 16, 2)])
def test_q8_0_rank_product_equals_f16_on_the_dequantised_weight(kind, a_mn, b_mn, M, K, nb, splits):
    """The DoRA products read the frozen Q8_0 weight through the rank-block kernel's converter
    warps (P = W A^T with W K-major; BD^T W as (W^T BD)^T with W MN-major).  Their f16 operand is
    exactly the bind-time dequantisation (fp32 d * q rounded to f16), so with the same split the
    result is bit-identical to the f16 kernel on that weight, and it matches the fp64 product."""
    from cases import q8_0_bytes
    rng = np.random.default_rng(M + 5 * K + nb)
    wshape = (K, M) if a_mn else (M, K)
    w = (0.02 * rng.standard_normal(wshape) * np.exp(rng.standard_normal((wshape[0], 1)))).astype(np.float32)
    blocks = q8_0_bytes(w)
    _, wh = A.q8_0_dequant(blocks)
    b = f16_bits(rng.standard_normal((K, nb) if b_mn else (nb, K)))
    c0 = rng.standard_normal((nb, M) if kind == A.RANK_ACC_T else (M, nb)).astype(np.float32)
    c8 = A.rank_gemm_q8_0(blocks, b, M, K, nb, a_mn, b_mn, kind, alpha=0.5, C_init=c0, splits=splits)
    c16 = A.rank_gemm_f16(wh.reshape(wshape), b, M, K, nb, a_mn, b_mn, kind, alpha=0.5, C_init=c0, splits=splits)
    np.testing.assert_array_equal(c8, c16)
    wf = bits_to_f32(wh).reshape(wshape).astype(np.float64)
    am = wf.T if a_mn else wf                                    # A(m, k) [M][K]
    bk = bits_to_f32(b).astype(np.float64)
    bm = bk if b_mn else bk.T                                    # B(k, n) [K][nb]
    ref = 0.5 * (am @ bm)
    ref = c0 + (ref.T if kind == A.RANK_ACC_T else ref)
    assert np.abs(c8 - ref).max() / np.abs(ref).max() < 1e-5
