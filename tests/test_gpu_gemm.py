"""Projection GEMM kernels vs numpy (f16 inputs are exact in fp32; fp32 accumulation)."""
import numpy as np
import pytest

import actrain as A
from f16util import bits_to_f32, f16_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", [0, 1, 2, 3, 4, 5],
                         ids=["auto", "mma", "tcgen05", "tcgen05_pair", "tcgen05_pair128", "tcgen05_pair_whole"])
@pytest.mark.parametrize("b_mn", [False, True], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 256, 128), (6000, 1024, 1024), (1000, 4096, 256),
                                   (130, 512, 4096), (1000, 384, 256),
                                   # stream-K on the 2-CTA path (more pair tiles than pairs, a mostly idle
                                   # last round, long reductions): 76 tiles; 80 tiles with ragged rows
                                   (4864, 1024, 2048), (5000, 1024, 2112)])
def test_gemm_matches_numpy(path, b_mn, M, N, K):
    # path 3 takes 256-wide pair tiles when N % 256 == 0, else 128-wide ones (N = 384)
    if path in (3, 4, 5) and M <= 128:
        pytest.skip("the 2-CTA kernel needs M > 128")
    rng = np.random.default_rng(M + N + K)
    a = f16_bits(rng.standard_normal((M, K)))
    b = f16_bits(rng.standard_normal((K, N) if b_mn else (N, K)))
    c = A.gemm_f16(a, b, M, N, K, b_mn, path)
    af, bf = bits_to_f32(a).astype(np.float64), bits_to_f32(b).astype(np.float64)
    ref = af @ (bf if b_mn else bf.T)
    err = np.abs(c - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err


@pytest.mark.parametrize("path", [0, 3, 4, 5], ids=["auto", "pair", "pair128", "pair_whole"])
@pytest.mark.parametrize("b_mn", [False, True], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(300, 256, 128), (6000, 1024, 1024), (1000, 4096, 256), (4864, 1024, 2048),
                                   (5000, 1024, 2112), (6000, 1024, 4096), (1000, 384, 256)])
def test_q8_0_gemm_equals_f16_gemm_on_the_dequantised_weight(path, b_mn, M, N, K):
    """Q8_0 weights stay quantised on the device; the converter warps' f16 operand is exactly the
    bind-time dequantisation (tools/ac-quantize.cpp:161 blocks, fp32 d * q rounded to f16), so the
    product is bit-identical to the f16 GEMM on that dequantised weight with the same tile schedule
    (stream-K splits included: 4864 x 1024 x 2048, 5000 x 1024 x 2112 and 6000 x 1024 x 4096 split
    tiles on the 256-wide pair path), and matches the fp64 product of the dequantised operands on
    every 2-CTA path."""
    from cases import q8_0_bytes
    if path == 3 and N % 256:
        pytest.skip("256-wide pair tiles need N % 256 == 0")
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    a = f16_bits(rng.standard_normal((M, K)))
    wshape = (K, N) if b_mn else (N, K)
    w = (0.02 * rng.standard_normal(wshape) * np.exp(rng.standard_normal((wshape[0], 1)))).astype(np.float32)
    blocks = q8_0_bytes(w)
    _, wh = A.q8_0_dequant(blocks)
    c8 = A.gemm_q8_0(a, blocks, M, N, K, b_mn, path)
    if path in (3, 4, 5):  # the same tile schedule on f16 weights (auto may pick the 1-CTA kernel for f16)
        c16 = A.gemm_f16(a, wh.reshape(wshape), M, N, K, b_mn, path)
        np.testing.assert_array_equal(c8, c16)
    wf = bits_to_f32(wh).reshape(wshape).astype(np.float64)
    ref = bits_to_f32(a).astype(np.float64) @ (wf if b_mn else wf.T)
    assert np.abs(c8 - ref).max() / np.abs(ref).max() < 1e-5
