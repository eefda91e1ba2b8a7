// Counter-based random numbers for on-device sampling: Philox4x32-10 (Salmon, Moraes, Dror and
// Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011) -- ten rounds of two 32x32->64
// multiplications on a 128-bit counter under a 64-bit key bumped by the Weyl constants between
// rounds -- and Box-Muller normals from its words.  Any (key, counter) gives the same four words
// on every thread, launch and device, so a draw is a pure function of the seed and the element's
// index: no generator state to carry between steps, and a resumed run draws what an
// uninterrupted one would.
#pragma once
#include <cstdint>

namespace act {

struct Philox4 {
    uint32_t v[4];
};

__host__ __device__ inline Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                 uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
    for (int r = 0; r < 10; ++r) {
        if (r) {
            k0 += W0;
            k1 += W1;
        }
        const uint64_t p0 = (uint64_t)M0 * c0, p1 = (uint64_t)M1 * c2;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
    }
    return Philox4{{c0, c1, c2, c3}};
}

// a word as a uniform in (0, 1]: the top 24 bits plus one, times 2^-24 (never 0, so its log is finite)
__host__ __device__ inline float philox_open01(uint32_t x) { return (float)((x >> 8) + 1) * (1.0f / 16777216.0f); }
// a word as a uniform in [0, 1)
__host__ __device__ inline float philox_01(uint32_t x) { return (float)(x >> 8) * (1.0f / 16777216.0f); }

}  // namespace act
