"""Projection GEMM kernels vs numpy (bf16 inputs are exact in fp32; fp32 accumulation)."""
import numpy as np
import pytest

import actrain as A

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bits_to_f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("path", [1, 2, 3], ids=["mma", "tcgen05", "tcgen05_pair"])
@pytest.mark.parametrize("b_mn", [False, True], ids=["NT", "NN"])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 256, 128), (6000, 1024, 1024), (1000, 4096, 256),
                                   (130, 512, 4096)])
def test_gemm_matches_numpy(path, b_mn, M, N, K):
    if path == 3 and (N % 256 or M <= 128):
        pytest.skip("the 2-CTA kernel needs N % 256 == 0 and M > 128")
    rng = np.random.default_rng(M + N + K)
    a = bf16_bits(rng.standard_normal((M, K)))
    b = bf16_bits(rng.standard_normal((K, N) if b_mn else (N, K)))
    c = A.gemm_bf16(a, b, M, N, K, b_mn, path)
    af, bf = bits_to_f32(a).astype(np.float64), bits_to_f32(b).astype(np.float64)
    ref = af @ (bf if b_mn else bf.T)
    err = np.abs(c - ref).max() / np.abs(ref).max()
    assert err < 1e-5, err
