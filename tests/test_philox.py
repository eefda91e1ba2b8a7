"""The counter-based generator behind on-device sampling (csrc/philox.cuh): Philox4x32-10 against
the published known-answer vectors of its authors' Random123 distribution, and the library's
header (compiled for the host) against this restatement."""
import os
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "audiocraft.cpp_b200", "csrc")

M0, M1, W0, W1 = 0xD2511F53, 0xCD9E8D57, 0x9E3779B9, 0xBB67AE85
MASK = 0xFFFFFFFF


def philox4x32_10(ctr, key):
    c0, c1, c2, c3 = ctr
    k0, k1 = key
    for r in range(10):
        if r:
            k0, k1 = (k0 + W0) & MASK, (k1 + W1) & MASK
        p0, p1 = M0 * c0, M1 * c2
        c0, c1, c2, c3 = ((p1 >> 32) ^ c1 ^ k0) & MASK, p1 & MASK, ((p0 >> 32) ^ c3 ^ k1) & MASK, p0 & MASK
    return c0, c1, c2, c3


KAT = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
       ((MASK, MASK, MASK, MASK), (MASK, MASK), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
       ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]


def test_known_answer_vectors():
    for ctr, key, want in KAT:
        assert philox4x32_10(ctr, key) == want


def box_muller(words):
    """The device's normals from one call's words (mf_sample_kernel), in fp64 for reference."""
    w = np.asarray(words, np.uint64)
    u_open = ((w[0::2] >> np.uint64(8)) + np.uint64(1)).astype(np.float64) / 16777216.0
    u = (w[1::2] >> np.uint64(8)).astype(np.float64) / 16777216.0
    rad = np.sqrt(-2.0 * np.log(u_open))
    return np.stack([rad * np.cos(2 * np.pi * u), rad * np.sin(2 * np.pi * u)], -1).reshape(-1)


PROGRAM = r"""
#include <cstdio>
#include "philox.cuh"
int main() {
    const unsigned v[][6] = {{0, 0, 0, 0, 0, 0}, {1, 2, 3, 4, 5, 6}, {0xffffffffu, 0, 7, 0x4d46, 0xdeadbeefu, 42}};
    for (auto& a : v) {
        const auto r = act::philox4x32_10(a[0], a[1], a[2], a[3], a[4], a[5]);
        std::printf("%u %u %u %u\n", r.v[0], r.v[1], r.v[2], r.v[3]);
    }
    std::printf("%a %a\n", act::philox_open01(0u), act::philox_01(0xffffffffu));
    return 0;
}
"""


def test_header_matches_the_restatement(tmp_path):
    src = tmp_path / "p.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "p"
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    if not os.path.exists(nvcc):
        pytest.skip("nvcc is not available")
    subprocess.run([nvcc, "-std=c++17", "-I" + CSRC, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    cases = [((0, 0, 0, 0), (0, 0)), ((1, 2, 3, 4), (5, 6)), ((MASK, 0, 7, 0x4D46), (0xDEADBEEF, 42))]
    for line, (ctr, key) in zip(out, cases):
        assert tuple(int(x) for x in line.split()) == philox4x32_10(ctr, key)
    lo, hi = (float.fromhex(x) for x in out[3].split())
    assert lo == 2.0 ** -24 and hi == 1.0 - 2.0 ** -24


def test_normals_have_unit_moments():
    words = [w for i in range(20000) for w in philox4x32_10((i, 3, 0, 0x4D46), (11, 0))]
    z = box_muller(words)
    assert abs(z.mean()) < 0.01 and abs(z.var() - 1) < 0.02
    assert abs(((z > 1.96) | (z < -1.96)).mean() - 0.05) < 0.005
