"""Python restatement of the C++ standard-library random draws the trainer front ends make
(GNU libstdc++, the library the reference CLIs are built with): std::mt19937, the float
generate_canonical, uniform_real_distribution<float>, normal_distribution<float> (Marsaglia polar,
one value cached), uniform_int_distribution (Lemire's nearly divisionless reduction for a 32-bit
engine) and std::shuffle (two swap positions per draw when the range allows).  logf / expf /
sqrtf come from the C library through ctypes, so the floats match bit for bit.

Test infrastructure: the CPU tests pin it against a compiled C++ program, and the GPU tests use
it to replay mf-train's draws for the oracle.
"""
import ctypes
import ctypes.util

import numpy as np

_libm = ctypes.CDLL(ctypes.util.find_library("m"))
for _f in ("logf", "expf", "sqrtf"):
    getattr(_libm, _f).restype = ctypes.c_float
    getattr(_libm, _f).argtypes = [ctypes.c_float]

F32 = np.float32


def logf(x):
    return F32(_libm.logf(float(x)))


def expf(x):
    return F32(_libm.expf(float(x)))


def sqrtf(x):
    return F32(_libm.sqrtf(float(x)))


class MT19937:
    """std::mt19937 (32-bit Mersenne Twister, seed by the standard linear recurrence)."""

    N, M = 624, 397

    def __init__(self, seed=5489):
        mt = [0] * self.N
        mt[0] = seed & 0xFFFFFFFF
        for i in range(1, self.N):
            mt[i] = (1812433253 * (mt[i - 1] ^ (mt[i - 1] >> 30)) + i) & 0xFFFFFFFF
        self.mt, self.i = mt, self.N

    def _twist(self):
        mt = self.mt
        for k in range(self.N):
            y = (mt[k] & 0x80000000) | (mt[(k + 1) % self.N] & 0x7FFFFFFF)
            v = mt[(k + self.M) % self.N] ^ (y >> 1)
            if y & 1:
                v ^= 0x9908B0DF
            mt[k] = v
        self.i = 0

    def __call__(self):
        if self.i >= self.N:
            self._twist()
        y = self.mt[self.i]
        self.i += 1
        y ^= y >> 11
        y ^= (y << 7) & 0x9D2C5680
        y ^= (y << 15) & 0xEFC60000
        y ^= y >> 18
        return y & 0xFFFFFFFF


def canonical(g):
    """generate_canonical<float, 24>: one 32-bit draw scaled by 2^-32, kept below 1."""
    r = F32(g()) / F32(4294967296.0)
    return F32(np.nextafter(F32(1), F32(0))) if r >= F32(1) else r


def uniform_real(g, a=0.0, b=1.0):
    return canonical(g) * (F32(b) - F32(a)) + F32(a)


class Normal:
    """normal_distribution<float>: polar method, the second value of each pair kept for the next call."""

    def __init__(self, mean=0.0, stddev=1.0):
        self.mean, self.stddev, self.saved = F32(mean), F32(stddev), None

    def __call__(self, g):
        if self.saved is not None:
            ret, self.saved = self.saved, None
        else:
            while True:
                x = F32(2) * canonical(g) - F32(1)
                y = F32(2) * canonical(g) - F32(1)
                r2 = x * x + y * y
                if not (r2 > 1 or r2 == 0):
                    break
            mult = sqrtf(F32(-2) * logf(r2) / r2)
            self.saved = x * mult
            ret = y * mult
        return ret * self.stddev + self.mean


def _nd32(g, rng):
    """Lemire's nearly divisionless reduction of a 32-bit draw to [0, rng) (rng < 2^32)."""
    product = g() * rng
    low = product & 0xFFFFFFFF
    if low < rng:
        threshold = (-rng) % (1 << 32) % rng
        while low < threshold:
            product = g() * rng
            low = product & 0xFFFFFFFF
    return product >> 32


def uniform_int(g, a, b):
    """uniform_int_distribution over [a, b] driven by a 32-bit engine."""
    urange = (b - a) & 0xFFFFFFFFFFFFFFFF
    if urange == 0xFFFFFFFF:
        return a + g()
    return a + _nd32(g, urange + 1)


def shuffle(seq, g):
    """std::shuffle: pairs of swap positions from one draw while the engine's range allows it."""
    n = len(seq)
    if n == 0:
        return
    if 0xFFFFFFFF // n >= n:
        i = 1
        if n % 2 == 0:
            j = uniform_int(g, 0, 1)
            seq[i], seq[j] = seq[j], seq[i]
            i += 1
        while i != n:
            b0 = i + 1
            x = uniform_int(g, 0, b0 * (b0 + 1) - 1)
            p0, p1 = x // (b0 + 1), x % (b0 + 1)
            seq[i], seq[p0] = seq[p0], seq[i]
            i += 1
            seq[i], seq[p1] = seq[p1], seq[i]
            i += 1
        return
    for i in range(1, n):
        j = uniform_int(g, 0, i)
        seq[i], seq[j] = seq[j], seq[i]


def time_sample(g, kind="uniform", mean=0.0, stddev=1.0):
    """MfTimeSampler::sample (src/mf/train.h:23-28)."""
    if kind == "uniform":
        return uniform_real(g, 0, 1)
    z = Normal(mean, stddev)(g)
    e = expf(-abs(z))
    v = F32(1) / (F32(1) + e) if z >= 0 else e / (F32(1) + e)
    return F32(min(max(v, F32(1e-6)), F32(1) - F32(1e-6)))
